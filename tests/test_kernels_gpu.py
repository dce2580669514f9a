"""Numerics of the bandwidth-bound kernels against float32 PyTorch references."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_rmsnorm_fwd_bwd(cuda_ext):
    torch.manual_seed(0)
    T, H = 257, 3584
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    r = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H, device="cuda")).to(torch.bfloat16)
    h = torch.empty_like(x)
    y = torch.empty_like(x)
    rstd = torch.empty(T, device="cuda")
    cuda_ext.rmsnorm_fwd(x, r, h, w, y, rstd, 1e-6)
    hf = x.float() + r.float()
    ref = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    torch.testing.assert_close(h.float(), hf, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)
    # backward
    hb = h.float().requires_grad_(True)
    wb = w.float().requires_grad_(True)
    out = hb * torch.rsqrt(hb.pow(2).mean(-1, keepdim=True) + 1e-6) * wb
    dy = torch.randn_like(x)
    out.backward(dy.float())
    dx = torch.empty_like(x)
    dw = torch.zeros(H, device="cuda")
    cuda_ext.rmsnorm_bwd(h, w, rstd, dy, None, dx, dw)
    torch.testing.assert_close(dx.float(), hb.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(dw, wb.grad, rtol=1e-2, atol=1e-1)


def _rope_ref(x, pos, inv_freq):
    ang = pos.float()[:, None] * inv_freq[None, :]  # [T, 64]
    cos = torch.cat([ang.cos(), ang.cos()], -1)[:, None, :]
    sin = torch.cat([ang.sin(), ang.sin()], -1)[:, None, :]
    x1, x2 = x[..., :64], x[..., 64:]
    rot = torch.cat([-x2, x1], -1)
    return x * cos + rot * sin


@pytest.mark.parametrize("qk_norm", [False, True])
def test_qk_norm_rope(cuda_ext, qk_norm):
    torch.manual_seed(0)
    T, nq, nk = 100, 4, 2
    W = (nq + 2 * nk) * 128
    qkv = torch.randn(T, W, device="cuda", dtype=torch.bfloat16)
    pos = torch.randint(0, 4096, (T,), device="cuda", dtype=torch.int32)
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, 128, 2, device="cuda").float() / 128))
    qw = (1 + 0.1 * torch.randn(128, device="cuda")).to(torch.bfloat16) if qk_norm else None
    kw = (1 + 0.1 * torch.randn(128, device="cuda")).to(torch.bfloat16) if qk_norm else None
    pre = qkv.clone()
    rstd = torch.empty(T * (nq + nk), device="cuda")
    cuda_ext.qk_norm_rope_fwd(qkv, nq, nk, pos, inv_freq, qw, kw, rstd, 1e-6)
    x = pre.float()[:, : (nq + nk) * 128].view(T, nq + nk, 128).requires_grad_(True)
    y = x
    if qk_norm:
        wcat = torch.stack([qw.float()] * nq + [kw.float()] * nk)[None]
        y = y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + 1e-6) * wcat
    ref = _rope_ref(y, pos, inv_freq)
    got = qkv[:, : (nq + nk) * 128].float().view(T, nq + nk, 128)
    torch.testing.assert_close(got, ref, rtol=2e-2, atol=3e-2)
    # v untouched
    assert torch.equal(qkv[:, (nq + nk) * 128 :], pre[:, (nq + nk) * 128 :])
    # backward
    g = torch.randn(T, nq + nk, 128, device="cuda")
    ref.backward(g)
    dq = torch.zeros(T, W, device="cuda", dtype=torch.bfloat16)
    dq[:, : (nq + nk) * 128] = g.view(T, -1).to(torch.bfloat16)
    dqw = torch.zeros(128, device="cuda")
    dkw = torch.zeros(128, device="cuda")
    cuda_ext.qk_norm_rope_bwd(dq, pre, nq, nk, pos, inv_freq, qw, kw, rstd, dqw, dkw)
    torch.testing.assert_close(dq[:, : (nq + nk) * 128].float().view(T, nq + nk, 128), x.grad, rtol=3e-2, atol=3e-2)


def test_swiglu(cuda_ext):
    torch.manual_seed(0)
    T, I = 64, 1024
    gu = torch.randn(T, 2 * I, device="cuda", dtype=torch.bfloat16)
    h = torch.empty(T, I, device="cuda", dtype=torch.bfloat16)
    cuda_ext.swiglu_fwd(gu, h)
    g = gu.float()[:, :I].requires_grad_(True)
    u = gu.float()[:, I:].requires_grad_(True)
    ref = torch.nn.functional.silu(g) * u
    torch.testing.assert_close(h.float(), ref, rtol=2e-2, atol=2e-2)
    dh = torch.randn(T, I, device="cuda", dtype=torch.bfloat16)
    ref.backward(dh.float())
    dgu = torch.empty_like(gu)
    cuda_ext.swiglu_bwd(gu, dh, dgu)
    torch.testing.assert_close(dgu[:, :I].float(), g.grad, rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(dgu[:, I:].float(), u.grad, rtol=3e-2, atol=3e-2)


def test_embedding(cuda_ext):
    V, H, T = 1000, 256, 300
    table = torch.randn(V, H, device="cuda", dtype=torch.bfloat16)
    ids = torch.randint(0, V, (T,), device="cuda")
    out = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)
    cuda_ext.embedding_fwd(table, ids, out)
    assert torch.equal(out, table[ids])
    dy = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    dt = torch.zeros(V, H, device="cuda")
    cuda_ext.embedding_bwd(dy, ids, dt)
    ref = torch.zeros(V, H, device="cuda").index_add_(0, ids, dy.float())
    torch.testing.assert_close(dt, ref, rtol=1e-4, atol=1e-4)


def test_adamw_matches_torch(cuda_ext):
    torch.manual_seed(0)
    n = 10_003
    p = torch.randn(n, device="cuda")
    p_ref = p.clone().requires_grad_(True)
    opt = torch.optim.AdamW([p_ref], lr=1e-2, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    p16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    for step in range(1, 4):
        g = torch.randn(n, device="cuda")
        p_ref.grad = g.clone() * 0.5
        opt.step()
        cuda_ext.adamw_step(p, g, m, v, p16, 1e-2, 0.9, 0.95, 1e-8, 0.1, step, None, 0.5)
    torch.testing.assert_close(p, p_ref.detach(), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(p16.float(), p, rtol=1e-2, atol=1e-2)


def test_sumsq_clip(cuda_ext):
    x = torch.randn(100_001, device="cuda")
    out = torch.zeros(2, device="cuda")
    cuda_ext.sumsq(x, out)
    torch.testing.assert_close(out[0], x.pow(2).sum(), rtol=1e-4, atol=1e-2)
    assert out[1].item() == 0
    f = torch.zeros(2, device="cuda")
    cuda_ext.clip_factor(out, 1.0, f)
    torch.testing.assert_close(f[1], x.norm(), rtol=1e-4, atol=1e-3)
    assert abs(f[0].item() - 1.0 / x.norm().item()) < 1e-4


@pytest.mark.parametrize("tau", [1.0, 0.7])
def test_softmax_stats_and_grad(cuda_ext, tau):
    torch.manual_seed(0)
    R, V = 37, 151936
    z = (torch.randn(R, V, device="cuda") * 3).to(torch.bfloat16)
    tgt = torch.randint(0, V, (R,), device="cuda")
    lse = torch.empty(R, device="cuda")
    lp = torch.empty(R, device="cuda")
    ent = torch.empty(R, device="cuda")
    cuda_ext.softmax_stats(z, tgt, 1.0 / tau, lse, lp, ent)
    zf = (z.float() / tau).requires_grad_(True)
    logp = torch.log_softmax(zf, -1)
    ref_lp = logp.gather(1, tgt[:, None])[:, 0]
    ref_ent = -(logp.exp() * logp).sum(-1)
    torch.testing.assert_close(lse, torch.logsumexp(zf, -1), rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(lp, ref_lp, rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(ent, ref_ent, rtol=1e-3, atol=1e-3)
    dlp = torch.randn(R, device="cuda")
    dent = torch.randn(R, device="cuda")
    zz = (z.float()).requires_grad_(True)
    lpp = torch.log_softmax(zz / tau, -1)
    (lpp.gather(1, tgt[:, None])[:, 0] * dlp + (-(lpp.exp() * lpp).sum(-1)) * dent).sum().backward()
    g = z.clone()
    cuda_ext.softmax_grad(g, tgt, 1.0 / tau, lse, ent, dlp, dent)
    torch.testing.assert_close(g.float(), zz.grad, rtol=5e-2, atol=1e-3)


@pytest.mark.parametrize("tau", [1.0, 0.7])
@pytest.mark.parametrize("V", [13, 4099, 151939])
def test_softmax_stats_ragged_vocab(cuda_ext, V, tau):
    """Vocabularies that are not a multiple of 8 (the scalar tail loop) and
    rows shorter than one pass of the block (fewer than 512 vectors): rows
    padded to a 16-byte stride, compared with torch logsumexp / entropy."""
    torch.manual_seed(V)
    R = 5
    ld = (V + 7) // 8 * 8
    buf = (torch.randn(R, ld, device="cuda") * 3).to(torch.bfloat16)
    z = buf[:, :V]
    tgt = torch.tensor([0, V - 1, V // 2, V - 2, 1], device="cuda")
    lse = torch.empty(R, device="cuda")
    lp = torch.empty(R, device="cuda")
    ent = torch.empty(R, device="cuda")
    cuda_ext.softmax_stats(z, tgt, 1.0 / tau, lse, lp, ent)
    zf = z.float() / tau
    logp = torch.log_softmax(zf, -1)
    torch.testing.assert_close(lse, torch.logsumexp(zf, -1), rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(lp, logp.gather(1, tgt[:, None])[:, 0], rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(ent, -(logp.exp() * logp).sum(-1), rtol=1e-3, atol=1e-3)
    # the padding columns were not read as logits
    buf2 = buf.clone()
    buf2[:, V:] = 1e4
    lse2 = torch.empty(R, device="cuda")
    cuda_ext.softmax_stats(buf2[:, :V], tgt, 1.0 / tau, lse2, None, None)
    torch.testing.assert_close(lse2, lse, rtol=0, atol=0)


def test_adamw8_kernel_matches_cpu_oracle(cuda_ext):
    """8-bit AdamW kernel against the float32 torch formulation of the same
    codes: parameters to float rounding, decoded moments within one code step
    (log2 / exp2 may round a boundary value to the neighbouring code)."""
    from wavelet_b200 import ops

    torch.manual_seed(0)
    n = 256 * 37 + 101  # a partial last block
    p = torch.randn(n) * 0.02
    m8 = torch.zeros(n, dtype=torch.int8)
    v8 = torch.zeros(n, dtype=torch.uint8)
    nb = (n + 255) // 256
    am, av = torch.zeros(nb), torch.zeros(nb)
    pd, m8d, v8d, amd, avd = (t.cuda() for t in (p.clone(), m8.clone(), v8.clone(), am.clone(), av.clone()))
    p16 = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    for step in range(1, 6):
        g = torch.randn(n) * torch.exp2(torch.randint(-8, 2, (n,)).float())
        kw = dict(lr=1e-2, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.1, step=step, gscale_host=0.5)
        ops.adamw8_flat_(p, g, m8, v8, am, av, None, **kw)
        ops.adamw8_flat_(pd, g.cuda(), m8d, v8d, amd, avd, p16, **kw)
        # re-sync the codes so the next step starts from the same state
        torch.testing.assert_close(pd.cpu(), p, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(amd.cpu(), am, rtol=1e-5, atol=0)
        dm = (m8d.cpu().int() - m8.int()).abs()
        dv = (v8d.cpu().int() - v8.int()).abs()
        assert int(dm.max()) <= 1 and int(dv.max()) <= 1
        assert float((dm > 0).float().mean()) < 0.01
        m8d.copy_(m8.cuda())
        v8d.copy_(v8.cuda())
        pd.copy_(p.cuda())
    torch.testing.assert_close(p16.float().cpu(), p.to(torch.bfloat16).float(), rtol=1e-2, atol=1e-4)
