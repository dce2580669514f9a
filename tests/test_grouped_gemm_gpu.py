"""Grouped (MoE expert) tcgen05 GEMM modes against float32 per-expert references."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _layout(counts, pad=128):
    padded = [(c + pad - 1) // pad * pad for c in counts]
    starts = [sum(padded[:i]) for i in range(len(counts))]
    tiles = [e for e in range(len(counts)) for _ in range(padded[e] // pad)]
    return padded, starts, tiles, sum(padded)


@pytest.mark.parametrize("counts", [[5, 130, 0, 260], [128, 1, 300]])
def test_grouped_modes(cuda_ext, counts):
    torch.manual_seed(0)
    E = len(counts)
    H, N = 256, 384
    padded, starts, tiles, R = _layout(counts)
    x = torch.zeros(R, H, device="cuda", dtype=torch.bfloat16)
    for e in range(E):
        x[starts[e] : starts[e] + counts[e]] = torch.randn(counts[e], H, device="cuda") / 4
    W = (torch.randn(E, N, H, device="cuda") / 16).to(torch.bfloat16)
    tg = torch.tensor(tiles, dtype=torch.int32, device="cuda")
    # mode 1, K-major B: y = x W_e^T
    y = torch.empty(R, N, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm_grouped(x, False, W.view(E * N, H), False, y, 1, R, N, H, tg, N, E * N, None, None, E, 0, 1.0)
    # mode 1, MN-major B (dgrad): dx = dy W_e
    dy = torch.zeros(R, N, device="cuda", dtype=torch.bfloat16)
    for e in range(E):
        dy[starts[e] : starts[e] + counts[e]] = torch.randn(counts[e], N, device="cuda") / 4
    dx = torch.empty(R, H, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm_grouped(dy, False, W.view(E * N, H), True, dx, 1, R, H, N, tg, N, E * N, None, None, E, 0, 1.0)
    # mode 2 (wgrad): dW_e += dy_e^T x_e
    dW = torch.ones(E * N, H, device="cuda", dtype=torch.float32)
    ks = torch.tensor(starts, dtype=torch.int32, device="cuda")
    kl = torch.tensor(padded, dtype=torch.int32, device="cuda")
    cuda_ext.gemm_grouped(dy, True, x, True, dW, 2, N, H, R, None, 0, 0, ks, kl, E, 2, 1.0)
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) == 0
    for e in range(E):
        s, c = starts[e], counts[e]
        if c == 0:
            assert torch.all(dW[e * N : (e + 1) * N] == 1)
            continue
        ref_y = x[s : s + c].float() @ W[e].float().t()
        torch.testing.assert_close(y[s : s + c].float(), ref_y, rtol=2e-2, atol=2e-2)
        ref_dx = dy[s : s + c].float() @ W[e].float()
        torch.testing.assert_close(dx[s : s + c].float(), ref_dx, rtol=2e-2, atol=2e-2)
        ref_dw = 1 + dy[s : s + c].float().t() @ x[s : s + c].float()
        torch.testing.assert_close(dW[e * N : (e + 1) * N], ref_dw, rtol=1e-3, atol=1e-2)
