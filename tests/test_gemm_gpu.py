"""Numerics of the tcgen05 GEMM against a float32 PyTorch reference."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, a_mn, b, b_mn):
    A = a.float().t() if a_mn else a.float()  # [M, K]
    B = b.float().t() if b_mn else b.float()  # [N, K]
    return A @ B.t()


@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("shape", [(128, 256, 64), (300, 520, 200), (1024, 768, 512), (77, 1000, 4096)])
def test_gemm_layouts(cuda_ext, a_mn, b_mn, shape):
    M, N, K = shape
    torch.manual_seed(0)
    dev = "cuda"
    a = torch.randn((K, M) if a_mn else (M, K), device=dev, dtype=torch.bfloat16)
    b = torch.randn((K, N) if b_mn else (N, K), device=dev, dtype=torch.bfloat16)
    if (a.shape[1] % 8) or (b.shape[1] % 8):
        pytest.skip("TMA needs 16-byte row pitch")
    ref = _ref(a, a_mn, b, b_mn)
    c = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    cuda_ext.gemm(a, a_mn, b, b_mn, c, cuda_ext.EPI_BF16, 1.0, None)
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) == 0
    err = (c.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 1e-2 * scale + 1e-2, (err, scale)


@pytest.mark.parametrize("epi", ["f32", "f32acc", "bias"])
def test_gemm_epilogues(cuda_ext, epi):
    torch.manual_seed(1)
    M, N, K = 256, 384, 320
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    ref = a.float() @ b.float().t()
    if epi == "f32":
        c = torch.empty(M, N, device="cuda", dtype=torch.float32)
        cuda_ext.gemm(a, False, b, False, c, cuda_ext.EPI_F32, 0.5, None)
        torch.testing.assert_close(c, 0.5 * ref, rtol=1e-3, atol=1e-2)
    elif epi == "f32acc":
        c = torch.ones(M, N, device="cuda", dtype=torch.float32)
        cuda_ext.gemm(a, False, b, False, c, cuda_ext.EPI_F32_ACC, 1.0, None)
        cuda_ext.gemm(a, False, b, False, c, cuda_ext.EPI_F32_ACC, 1.0, None)
        torch.testing.assert_close(c, 1 + 2 * ref, rtol=1e-3, atol=2e-2)
    else:
        bias = torch.randn(N, device="cuda", dtype=torch.bfloat16)
        c = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        cuda_ext.gemm(a, False, b, False, c, cuda_ext.EPI_BF16, 1.0, bias)
        torch.testing.assert_close(c.float(), ref + bias.float(), rtol=2e-2, atol=2e-1)
    assert cuda_ext.read_error(0) == 0


def test_gemm_large_k_persistent(cuda_ext):
    """More tiles than SMs so every CTA loops over several tiles and both TMEM buffers."""
    torch.manual_seed(2)
    M, N, K = 4096, 4096, 1024
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16) / 8
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / 8
    c = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm(a, False, b, False, c, cuda_ext.EPI_BF16, 1.0, None)
    ref = a.float() @ b.float().t()
    err = (c.float() - ref).abs().max().item()
    assert err < 0.05, err


@pytest.mark.parametrize("case", ["fwd_res", "wgrad_acc"])
def test_gemm_tail_split(cuda_ext, case):
    """Long-K shapes whose last wave is small (448 tiles on 148 SMs; 504
    tiles) run the tail tiles as K-pieces reduced by the last piece; repeated
    calls reuse the per-device tickets and workspace."""
    torch.manual_seed(3)
    dev = "cuda"
    if case == "fwd_res":
        M, N, K = 4096, 3584, 18944
        a = torch.randn(M, K, device=dev, dtype=torch.bfloat16) / 8
        b = torch.randn(N, K, device=dev, dtype=torch.bfloat16) / 8
        res = torch.randn(M, N, device=dev, dtype=torch.bfloat16)
        ref = a.float() @ b.float().t() + res.float()
        from wavelet_b200 import ops

        for _ in range(2):
            c = ops.gemm(a, b, res=res)
            torch.cuda.synchronize()
            err = (c.float() - ref).abs().max().item()
            assert err <= 1e-2 * ref.abs().max().item() + 2e-2, err
    else:
        M, N, K = 4608, 3584, 16384  # wgrad: C[M, N] += A^T B with MN-major A [K, M], B [K, N]
        a = torch.randn(K, M, device=dev, dtype=torch.bfloat16) / 8
        b = torch.randn(K, N, device=dev, dtype=torch.bfloat16) / 8
        c = torch.ones(M, N, device=dev, dtype=torch.float32)
        for _ in range(2):
            cuda_ext.gemm(a, True, b, True, c, cuda_ext.EPI_F32_ACC, 1.0, None)
        torch.cuda.synchronize()
        ref = 1 + 2 * (a.float().t() @ b.float())
        torch.testing.assert_close(c, ref, rtol=1e-3, atol=5e-2)
    assert cuda_ext.read_error(0) == 0
