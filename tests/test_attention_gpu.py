"""tcgen05 varlen causal attention (forward and backward) against a float32
PyTorch reference, including GQA and sequence lengths that are not multiples
of the 128-row tile."""

import math

import pytest
import torch

from wavelet_b200.ops import reference as ref
from wavelet_b200.ops.attention import attention_bwd, attention_fwd, native_attention

pytestmark = pytest.mark.gpu


def _ref_fwd_bwd(q, k, v, cu, do):
    qf = q.float().requires_grad_(True)
    kf = k.float().requires_grad_(True)
    vf = v.float().requires_grad_(True)
    out = ref.attention(qf, kf, vf, cu.cpu(), True)
    out.backward(do.float())
    return out.detach(), qf.grad, kf.grad, vf.grad


@pytest.mark.parametrize("lens,hq,hk", [([128], 2, 1), ([300, 77, 256], 4, 2), ([1000], 8, 2), ([5, 129, 640], 2, 2)])
def test_attention_matches_reference(cuda_ext, lens, hq, hk):
    assert native_attention()
    torch.manual_seed(0)
    T = sum(lens)
    W = (hq + 2 * hk) * 128
    qkv = torch.randn(T, W, device="cuda", dtype=torch.bfloat16)
    q = qkv[:, : hq * 128].view(T, hq, 128)
    k = qkv[:, hq * 128 : (hq + hk) * 128].view(T, hk, 128)
    v = qkv[:, (hq + hk) * 128 :].view(T, hk, 128)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device="cuda")
    out, lse = attention_fwd(q, k, v, cu, max(lens), True)
    do = torch.randn(T, hq, 128, device="cuda", dtype=torch.bfloat16)
    dq, dk, dv = attention_bwd(do, q, k, v, out, lse, cu, max(lens), True)
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) == 0
    ro, rdq, rdk, rdv = _ref_fwd_bwd(q, k, v, cu, do)
    torch.testing.assert_close(out.float(), ro, rtol=2e-2, atol=2e-2)
    # lse check
    for (s, e) in zip(cu[:-1].tolist(), cu[1:].tolist()):
        qs = q[s:e].float().transpose(0, 1)
        ks = k[s:e].float().transpose(0, 1).repeat_interleave(hq // hk, 0)
        sc = (qs @ ks.transpose(-1, -2)) / math.sqrt(128)
        L = e - s
        sc = sc.masked_fill(~torch.ones(L, L, dtype=torch.bool, device="cuda").tril(), float("-inf"))
        torch.testing.assert_close(lse[:, s:e], torch.logsumexp(sc, -1), rtol=1e-3, atol=1e-2)
    for got, want, name in ((dq, rdq, "dq"), (dk, rdk, "dk"), (dv, rdv, "dv")):
        err = (got.float() - want).abs().max().item()
        scale = want.abs().max().item()
        assert err <= 3e-2 * scale + 3e-2, (name, err, scale)


@pytest.mark.parametrize("lq,lk,hq,hk", [([128, 256], [256, 512], 4, 2), ([300, 64], [428, 448], 8, 2),
                                         ([128], [128], 2, 2), ([0, 200], [256, 456], 2, 1)])
def test_attention_separate_keys(cuda_ext, lq, lk, hq, hk):
    """Separate key sequences (context parallelism): the queries of sequence i
    are the last lq[i] of its lk[i] keys (offset a multiple of 128); keys that
    no query sees get zero gradients."""
    torch.manual_seed(1)
    Tq, Tk = sum(lq), sum(lk)
    q = torch.randn(Tq, hq, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(Tk, hk, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(Tk, hk, 128, device="cuda", dtype=torch.bfloat16)
    cuq = torch.tensor([0] + list(torch.tensor(lq).cumsum(0)), dtype=torch.int32, device="cuda")
    cuk = torch.tensor([0] + list(torch.tensor(lk).cumsum(0)), dtype=torch.int32, device="cuda")
    out, lse = attention_fwd(q, k, v, cuq, max(lq), True, None, cuk, max(lk))
    do = torch.randn(Tq, hq, 128, device="cuda", dtype=torch.bfloat16)
    dq, dk, dv = attention_bwd(do, q, k, v, out, lse, cuq, max(lq), True, None, cuk, max(lk))
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) == 0
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    ro = ref.attention(qf, kf, vf, cuq.cpu(), True, None, cuk.cpu())
    ro.backward(do.float())
    torch.testing.assert_close(out.float(), ro.detach(), rtol=2e-2, atol=2e-2)
    for got, want, name in ((dq, qf.grad, "dq"), (dk, kf.grad, "dk"), (dv, vf.grad, "dv")):
        err = (got.float() - want).abs().max().item()
        scale = want.abs().max().item()
        assert err <= 3e-2 * scale + 3e-2, (name, err, scale)
