"""Out-of-bounds write detection without compute-sanitizer: every output
below is a view in the middle of a larger buffer whose head and tail hold a
sentinel; after the kernel runs, the sentinels must be untouched.  Shapes
include partial tiles, the GEMM tail split and GQA attention."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

PAD = 8192
SENT = {torch.bfloat16: -12288.0, torch.float32: -3.0e38}


def padded(shape, dtype):
    n = math.prod(shape)
    buf = torch.full((PAD + n + PAD,), SENT[dtype], dtype=dtype, device="cuda")
    return buf, buf[PAD:PAD + n].view(shape)


def intact(buf, shape) -> bool:
    n = math.prod(shape)
    s = torch.full((PAD,), SENT[buf.dtype], dtype=buf.dtype, device="cuda")
    return torch.equal(buf[:PAD], s) and torch.equal(buf[PAD + n:], s)


@pytest.mark.parametrize("M,N,K", [(300, 520, 200), (77, 1000, 4096), (4096, 3584, 8192)])
def test_gemm_writes_stay_in_bounds(cuda_ext, M, N, K):
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16) / 8
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / 8
    buf, c = padded((M, N), torch.bfloat16)
    cuda_ext.gemm(a, False, b, False, c, cuda_ext.EPI_BF16, 1.0, None)
    dy = torch.randn(M, N, device="cuda", dtype=torch.bfloat16) / 8
    fbuf, f = padded((N, K), torch.float32)
    f.zero_()
    cuda_ext.gemm(dy, True, a, True, f, cuda_ext.EPI_F32_ACC, 1.0, None)  # weight-gradient layout: dy^T a
    torch.cuda.synchronize()
    assert intact(buf, (M, N)) and intact(fbuf, (N, K))
    assert cuda_ext.read_error(0) == 0


def test_attention_writes_stay_in_bounds(cuda_ext):
    from wavelet_b200.ops.attention import attention_fwd

    lens = [300, 77, 256]
    T, hq, hk = sum(lens), 8, 2
    q = torch.randn(T, hq, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(T, hk, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(T, hk, 128, device="cuda", dtype=torch.bfloat16)
    cu = torch.tensor([0, 300, 377, 633], dtype=torch.int32, device="cuda")
    obuf, out = padded((T, hq, 128), torch.bfloat16)
    lbuf, lse = padded((hq, T), torch.float32)
    cuda_ext.attn_fwd(q, k, v, cu, max(lens), True, 128 ** -0.5, out, lse, None, 0)
    ref, _ = attention_fwd(q, k, v, cu, max(lens), True)
    do = torch.randn_like(out)
    bufs = [padded(t.shape, torch.bfloat16) for t in (q, k, v)]
    cuda_ext.attn_bwd(do, q, k, v, out, lse, cu, max(lens), True, 128 ** -0.5, bufs[0][1], bufs[1][1], bufs[2][1],
                      None, 0)
    torch.cuda.synchronize()
    assert intact(obuf, out.shape) and intact(lbuf, lse.shape)
    assert all(intact(b, t.shape) for (b, _), t in zip(bufs, (q, k, v)))
    torch.testing.assert_close(out, ref, rtol=0, atol=0)
    assert cuda_ext.read_error(0) == 0


def test_elementwise_writes_stay_in_bounds(cuda_ext):
    rows, H, I = 517, 3584, 1000
    x = torch.randn(rows, H, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(H, device="cuda", dtype=torch.bfloat16)
    ybuf, y = padded((rows, H), torch.bfloat16)
    rbuf, rstd = padded((rows,), torch.float32)
    cuda_ext.rmsnorm_fwd(x, None, None, w, y, rstd, 1e-6)
    dy = torch.randn_like(x)
    dxbuf, dx = padded((rows, H), torch.bfloat16)
    dwbuf, dw = padded((H,), torch.float32)
    dw.zero_()
    cuda_ext.rmsnorm_bwd(x, w, rstd, dy, None, dx, dw)
    gu = torch.randn(rows, 2 * I, device="cuda", dtype=torch.bfloat16)
    hbuf, h = padded((rows, I), torch.bfloat16)
    cuda_ext.swiglu_fwd(gu, h)
    gbuf, dgu = padded((rows, 2 * I), torch.bfloat16)
    cuda_ext.swiglu_bwd(gu, torch.randn_like(h), dgu)
    table = torch.randn(1000, H, device="cuda", dtype=torch.bfloat16)
    ids = torch.randint(0, 1000, (rows,), device="cuda")
    ebuf, e = padded((rows, H), torch.bfloat16)
    cuda_ext.embedding_fwd(table, ids, e)
    torch.cuda.synchronize()
    for b, t in ((ybuf, y), (rbuf, rstd), (dxbuf, dx), (dwbuf, dw), (hbuf, h), (gbuf, dgu), (ebuf, e)):
        assert intact(b, t.shape)
    assert cuda_ext.read_error(0) == 0


def test_decode_and_row_kernels_stay_in_bounds(cuda_ext):
    B, Hq, Hk, bs, ctx = 5, 8, 2, 64, 300
    nb = -(-(ctx + 1) // bs)
    kc = torch.randn(B * nb + 1, Hk, bs, 128, device="cuda", dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    bt = torch.arange(B * nb, dtype=torch.int32, device="cuda").view(B, nb)
    cl = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    q = torch.randn(B, Hq, 128, device="cuda", dtype=torch.bfloat16)
    obuf, out = padded((B, Hq, 128), torch.bfloat16)
    cuda_ext.decode_attention(q, kc, vc, bt, cl, out, 2, 128 ** -0.5)
    # weighted gather-sum of rows (one-rank "peer" pointer = this buffer)
    T, k, H = 100, 4, 256
    src = torch.randn(400, H, device="cuda", dtype=torch.bfloat16)
    rank = torch.zeros(T * k, dtype=torch.int32, device="cuda")
    row = torch.randint(0, 400, (T * k,), device="cuda")
    wts = torch.rand(T * k, device="cuda")
    gbuf, g = padded((T, H), torch.bfloat16)
    cuda_ext.rows_gather_sum([src.data_ptr()], 1, H, rank, row, wts, k, None, g)
    sbuf, s = padded((T * H,), torch.bfloat16)
    slots = torch.randn(2 * T * H, device="cuda", dtype=torch.bfloat16)
    cuda_ext.slots_sum(slots, 2, T * H, T * H, None, s)
    torch.cuda.synchronize()
    assert intact(obuf, out.shape) and intact(gbuf, g.shape) and intact(sbuf, s.shape)
    assert cuda_ext.read_error(0) == 0
