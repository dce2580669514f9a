"""NF4 table, quantiser and CPU GEMM path (no GPU)."""

import torch

from wavelet_b200 import ops
from wavelet_b200.ops.nf4 import dequantize, nf4_table, quantize


def test_nf4_table_matches_published_values():
    # QLoRA paper (Dettmers et al. 2023), appendix: the NF4 data type values
    published = [-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453, -0.28444138169288635,
                 -0.18477343022823334, -0.09105003625154495, 0.0, 0.07958029955625534, 0.16093020141124725,
                 0.24611230194568634, 0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
                 0.7229568362236023, 1.0]
    for a, b in zip(nf4_table(), published):
        assert abs(a - b) < 1e-6


def test_quantize_roundtrip_nearest_code():
    torch.manual_seed(0)
    w = torch.randn(64, 256) * 0.02
    q = quantize(w)
    d = dequantize(q, torch.float32)
    lut = torch.tensor(nf4_table())
    blk = w.reshape(-1, 64)
    am = blk.abs().amax(1, keepdim=True)
    nearest = lut[(blk / am).unsqueeze(-1).sub(lut).abs().argmin(-1)] * am
    torch.testing.assert_close(d.reshape(-1, 64), nearest)
    # the block maximum is exact
    assert torch.allclose(d.reshape(-1, 64).abs().amax(1), am.squeeze(1))
    assert q.codes.dtype == torch.uint8 and q.codes.numel() == w.numel() // 2


def test_gemm_nf4_and_dual_cpu():
    torch.manual_seed(1)
    w = torch.randn(96, 128) * 0.05
    q = quantize(w)
    x = torch.randn(7, 128)
    u, lb = torch.randn(7, 64), torch.randn(96, 64)
    y = ops.gemm(x, q, a2=u, b2=lb)
    torch.testing.assert_close(y, x @ dequantize(q, torch.float32).t() + u @ lb.t(), rtol=1e-5, atol=1e-5)
