"""LoRA-fused (second operand pair) and NF4-B tcgen05 GEMM paths against
float32 references of the same math."""

import pytest
import torch

from wavelet_b200 import ops
from wavelet_b200.ops.nf4 import dequantize, nf4_table, quantize

pytestmark = pytest.mark.gpu


def _close(got, want, tol=2e-2):
    err = (got.float() - want).abs().max().item()
    scale = want.abs().max().item() + 1e-6
    assert err <= tol * scale, (err, scale)


@pytest.mark.parametrize("M,N,K,K2", [(300, 512, 384, 64), (128, 200, 256, 128)])
def test_dual_operand_forward_and_dgrad(cuda_ext, M, N, K, K2):
    torch.manual_seed(0)
    bf = torch.bfloat16
    x = torch.randn(M, K, device="cuda", dtype=bf)
    w = (torch.randn(N, K, device="cuda") / 16).to(bf)
    u = torch.randn(M, K2, device="cuda", dtype=bf)
    lb = (torch.randn(N, K2, device="cuda") / 8).to(bf)
    res = torch.randn(M, N, device="cuda", dtype=bf)
    y = ops.gemm(x, w, a2=u, b2=lb, res=res)
    _close(y, x.float() @ w.float().t() + u.float() @ lb.float().t() + res.float())
    # dgrad form: dx = dy W + g A  (B operands MN-major)
    dy = torch.randn(M, N, device="cuda", dtype=bf)
    g = torch.randn(M, K2, device="cuda", dtype=bf)
    la = (torch.randn(K2, K, device="cuda") / 8).to(bf)
    dx = ops.gemm(dy, w, b_mn=True, a2=g, b2=la)
    _close(dx, dy.float() @ w.float() + g.float() @ la.float())
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) == 0


@pytest.mark.parametrize("M,N,K", [(256, 512, 384), (333, 320, 192), (4096, 3584, 1024)])
def test_nf4_gemm(cuda_ext, M, N, K):
    torch.manual_seed(1)
    bf = torch.bfloat16
    w = torch.randn(N, K, device="cuda") * 0.02
    q = quantize(w)
    wd = dequantize(q, torch.float32)
    x = torch.randn(M, K, device="cuda", dtype=bf)
    y = ops.gemm(x, q)
    _close(y, x.float() @ wd.to(bf).float().t())
    # dgrad: dx = dy W  with W NF4 [N, K] read MN-major
    dy = torch.randn(M, N, device="cuda", dtype=bf)
    dx = ops.gemm(dy, q, b_mn=True)
    _close(dx, dy.float() @ wd.to(bf).float())
    # NF4 + LoRA second operand
    u = torch.randn(M, 64, device="cuda", dtype=bf)
    lb = (torch.randn(N, 64, device="cuda") / 8).to(bf)
    y2 = ops.gemm(x, q, a2=u, b2=lb)
    _close(y2, x.float() @ wd.to(bf).float().t() + u.float() @ lb.float().t())
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) == 0




def test_nf4_dequant_kernel_and_large_m_path(cuda_ext):
    from wavelet_b200.ops.nf4 import dequant_cache

    torch.manual_seed(2)
    w = torch.randn(384, 512, device="cuda") * 0.03
    q = quantize(w)
    ref = dequantize(q, torch.float32).to(torch.bfloat16)
    got = dequant_cache().get(q)
    assert torch.equal(got, ref)
    x = torch.randn(1024, 512, device="cuda", dtype=torch.bfloat16)  # M > FUSED_MAX_M: cached dense path
    _close(ops.gemm(x, q), x.float() @ ref.float().t())
    dy = torch.randn(1024, 384, device="cuda", dtype=torch.bfloat16)
    _close(ops.gemm(dy, q, b_mn=True), dy.float() @ ref.float())


@pytest.mark.parametrize("M,N,K", [(512, 2560, 9728), (64, 4096, 4096), (300, 1024, 3584)])
def test_splitk_skinny_gemm(cuda_ext, M, N, K):
    from wavelet_b200.ops import _splitk

    torch.manual_seed(3)
    bf = torch.bfloat16
    x = torch.randn(M, K, device="cuda", dtype=bf)
    w = (torch.randn(N, K, device="cuda") / 32).to(bf)
    bias = torch.randn(N, device="cuda", dtype=bf)
    res = torch.randn(M, N, device="cuda", dtype=bf)
    out = torch.empty(M, N, device="cuda", dtype=bf)
    assert _splitk(M, N, K, False, 0, out) > 1
    y = ops.gemm(x, w, bias=bias, res=res, alpha=0.5)
    _close(y, 0.5 * (x.float() @ w.float().t()) + bias.float() + res.float())
    dy = torch.randn(M, N, device="cuda", dtype=bf)
    w2 = (torch.randn(N, K, device="cuda") / 32).to(bf)
    dx = ops.gemm(dy, w2, b_mn=True)  # dgrad form (N=K output), split when skinny
    _close(dx, dy.float() @ w2.float())
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) == 0
