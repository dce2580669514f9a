"""Generator kernels and the native generator on the GPU.

* paged decode attention (split-K + combine) and KV append against a float32
  dense attention over the gathered cache;
* the sampler: greedy = argmax with the exact log-softmax, and a chi-square
  check of temperature sampling on a small vocabulary;
* the generator (CUDA-graph windowed decode and the eager path): its returned
  log-probs match teacher-forced log-probs of the training forward.
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("splits", [1, 4])
def test_decode_attention_and_kv_append(cuda_ext, splits):
    torch.manual_seed(0)
    B, Hq, Hk, D, bs, nblk = 5, 8, 2, 128, 64, 40
    kc = torch.zeros(nblk, Hk, bs, D, device="cuda", dtype=torch.bfloat16)  # head-major pages
    vc = torch.zeros_like(kc)
    lens = [1, 63, 64, 130, 300]
    perm = torch.randperm(nblk).tolist()
    bt = torch.zeros(B, 8, dtype=torch.int32)
    K, V, used = [], [], 0
    for i, L in enumerate(lens):
        nb = (L + bs - 1) // bs
        bt[i, :nb] = torch.tensor(perm[used : used + nb])
        used += nb
        k = torch.randn(L, Hk, D, device="cuda", dtype=torch.bfloat16)
        v = torch.randn(L, Hk, D, device="cuda", dtype=torch.bfloat16)
        slots = torch.tensor([int(bt[i, p // bs]) * bs + p % bs for p in range(L)], dtype=torch.int32, device="cuda")
        cuda_ext.kv_append(k, v, kc, vc, slots)
        K.append(k)
        V.append(v)
    q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(q)
    scale = 1 / math.sqrt(D)
    cuda_ext.decode_attention(q, kc, vc, bt.cuda(), torch.tensor(lens, dtype=torch.int32, device="cuda"), out, splits,
                              scale)
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) == 0
    rep = Hq // Hk
    for i, L in enumerate(lens):
        k = K[i].float().repeat_interleave(rep, 1)  # [L, Hq, D]
        v = V[i].float().repeat_interleave(rep, 1)
        s = torch.einsum("hd,lhd->hl", q[i].float(), k) * scale
        ref = torch.einsum("hl,lhd->hd", torch.softmax(s, -1), v)
        torch.testing.assert_close(out[i].float(), ref, rtol=2e-2, atol=2e-2)


def test_sampler_greedy_and_distribution(cuda_ext):
    torch.manual_seed(1)
    B, V = 4, 1000
    z = (torch.randn(B, V, device="cuda") * 3).to(torch.bfloat16)
    tok = torch.empty(B, dtype=torch.long, device="cuda")
    lp = torch.empty(B, dtype=torch.float32, device="cuda")
    cuda_ext.sample_tokens(z, torch.zeros(B, device="cuda"), None, 0.0, 0, None, tok, lp)
    assert torch.equal(tok, z.float().argmax(-1))
    torch.testing.assert_close(lp, torch.log_softmax(z.float(), -1).gather(1, tok[:, None])[:, 0], rtol=1e-4, atol=1e-4)
    # temperature 1 over a 8-token vocabulary: chi-square against softmax
    R, Vs = 20000, 8
    zs = torch.tensor([2.0, 1.0, 0.5, 0.0, -0.5, -1.0, 1.5, 0.2]).to(torch.bfloat16)
    zz = zs[None].expand(R, Vs).contiguous().cuda()
    t2 = torch.empty(R, dtype=torch.long, device="cuda")
    l2 = torch.empty(R, dtype=torch.float32, device="cuda")
    rows = torch.arange(R, dtype=torch.long, device="cuda")
    seed = torch.tensor([12345], dtype=torch.long, device="cuda")
    cuda_ext.sample_tokens(zz, torch.ones(R, device="cuda"), None, 0.0, 0, rows, t2, l2, seed)
    p = torch.softmax(zs.float(), -1)
    counts = torch.bincount(t2.cpu(), minlength=Vs).float()
    chi2 = ((counts - R * p) ** 2 / (R * p)).sum().item()
    assert chi2 < 30.0, chi2  # 7 degrees of freedom; p < 1e-4 above ~29
    torch.testing.assert_close(l2.cpu(), torch.log_softmax(zs.float(), -1)[t2.cpu()], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("graphs", [True, False])
def test_generator_logprobs_match_training_forward(cuda_ext, graphs):
    from wavelet_b200.inference.engine import Generator, SamplingParams
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.ops import lm_head

    cfg = PRESETS["tiny-gpu"]
    m = build_model(cfg, "cuda", torch.bfloat16, seed=5, with_grad=False, with_optimizer=False)
    gen = Generator(m, max_num_seqs=64, max_model_len=512, kv_cache_bytes=256 << 20, cuda_graphs=graphs)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(3, cfg.vocab_size, (L,), generator=g).tolist() for L in (5, 17, 64, 100)]
    params = SamplingParams(temperature=1.0, max_tokens=70, n=2, seed=3)
    if not graphs:
        gen._fast_ok = lambda seqs: False  # eager per-step path
    outs = gen.generate(prompts, params)
    assert len(outs) == 8 and all(len(o.token_ids) == 70 for o in outs)
    ids = [o.prompt_ids + o.token_ids for o in outs]
    lens = [len(x) for x in ids]
    flat = torch.tensor([t for x in ids for t in x], device="cuda")
    cu = torch.zeros(len(ids) + 1, dtype=torch.int32)
    cu[1:] = torch.tensor(lens).cumsum(0)
    pos = torch.cat([torch.arange(L, dtype=torch.int32) for L in lens]).cuda()
    with torch.no_grad():
        h = m.hidden(flat, m.batch_ctx(pos, cu.cuda(), max(lens)))
        tgt = torch.cat([flat[1:], flat[:1]])
        lp, _ = lm_head.logprob_entropy(h, m.head_weight(), tgt, 1.0, want_entropy=False)
    worst = 0.0
    for i, o in enumerate(outs):
        start = int(cu[i]) + len(o.prompt_ids) - 1
        ref = lp[start : start + len(o.token_ids)].cpu()
        worst = max(worst, (ref - torch.tensor(o.logprobs)).abs().max().item())
    assert worst < 0.1, worst


def test_sample_thresholds_kernel_matches_sort_oracle(cuda_ext):
    """Device top-k / top-p thresholds: top-k is the exact k-th largest logit;
    top-p is the logit at which the descending cumulative probability first
    reaches p (the kept mass reaches p, the mass strictly above does not), on
    bf16 rows with many tied values and mixed temperatures."""
    from wavelet_b200.inference.engine import sampling_thresholds_reference

    torch.manual_seed(0)
    B, V = 9, 151936
    z = (torch.randn(B, V, device="cuda") * 2.5).to(torch.bfloat16)
    z[3, :100] = 30.0  # a block of ties at the top
    top_k = [0, 1, 50, 120, 0, 0, 40, 3, 0]
    top_p = [1.0, 1.0, 1.0, 0.9, 0.5, 0.95, 0.7, 1.0, 0.999]
    inv_tau = torch.tensor([1.0, 1.0, 0.5, 1.0, 2.0, 1.0, 1.0 / 0.7, 1.0, 1.0], device="cuda")
    out = torch.empty(B, device="cuda")
    cuda_ext.sample_thresholds(z, torch.tensor(top_k, dtype=torch.int32, device="cuda"),
                               torch.tensor(top_p, device="cuda"), inv_tau, out)
    ref = sampling_thresholds_reference(z, top_k, top_p, inv_tau)
    zf = z.float()
    for i in range(B):
        if top_k[i] == 0 and top_p[i] >= 1.0:
            assert out[i].item() == float("-inf")
            continue
        if top_p[i] >= 1.0:
            assert out[i].item() == ref[i].item(), (i, out[i].item(), ref[i].item())
            continue
        pr = torch.softmax(zf[i] * inv_tau[i], -1)
        th = out[i].item()
        kth = float(torch.topk(zf[i], top_k[i]).values[-1]) if top_k[i] > 0 else float("-inf")
        pth = th if th > kth else None
        if pth is not None:  # the nucleus decides: kept mass >= p, mass strictly above < p
            assert float(pr[zf[i] >= pth].sum()) >= top_p[i] - 1e-4
            assert float(pr[zf[i] > pth].sum()) < top_p[i] + 1e-4
        assert abs(th - ref[i].item()) <= 0.0625 * max(1.0, abs(ref[i].item())), (i, th, ref[i].item())
