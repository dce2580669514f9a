"""Sampling-support replay of the trainer log-prob against the cases the
reference's chunked LM-head tests pin (tests/test_chunked_lm_head.py of the
reference): tokens outside the support never enter the exponent, rows with a
support renormalise over it only (forward and backward, head gradient into an
fp32 buffer), rows without one use the full vocabulary."""

import torch

from wavelet_b200.ops import reference as ref
from wavelet_b200.ops.support_head import SupportLogZ


def _support_lp(h, W, gW, tgt, supports, temperature):
    """Per-token log-prob: full softmax, replaced on rows with a support set."""
    lp, _ = ref.logprob_entropy(h @ W.t(), tgt, temperature)
    rows = [i for i, s in enumerate(supports) if s]
    if not rows:
        return lp
    K = max(len(supports[i]) for i in rows)
    ids = torch.full((len(rows), K), -1, dtype=torch.long)
    for r, i in enumerate(rows):
        ids[r, : len(supports[i])] = torch.tensor(supports[i])
    ridx = torch.tensor(rows)
    anchor = torch.empty(0, requires_grad=True)
    logz = SupportLogZ.apply(h, ridx, ids.clamp_min(0), ids >= 0, W, gW, temperature, anchor)
    zt = SupportLogZ.target_logit(h, ridx, tgt, W, gW, temperature, anchor)
    return lp.index_put((ridx,), zt - logz)


def test_support_excludes_large_logits_before_exp():
    V = 8201
    for excluded in (0, 8192):
        W = torch.zeros(V, 1)
        W[excluded] = 100.0
        h = torch.ones(1, 1, requires_grad=True)
        gW = torch.zeros(V, 1)
        lp = _support_lp(h, W, gW, torch.tensor([1]), [[1]], 1.0)
        lp.sum().backward()
        torch.testing.assert_close(lp, torch.zeros(1))
        torch.testing.assert_close(h.grad, torch.zeros_like(h))
        torch.testing.assert_close(gW, torch.zeros_like(gW))


def test_support_forward_and_backward_match_masked_full_softmax():
    torch.manual_seed(4)
    V, H, T, tau = 9, 5, 4, 0.9
    h = torch.randn(T, H, requires_grad=True)
    W = torch.randn(V, H)
    tgt = torch.tensor([1, 4, 2, 8])
    supports = [[1, 3, 7], [0, 4], [], [8]]
    gW = torch.zeros(V, H)
    lp = _support_lp(h, W, gW, tgt, supports, tau)
    lp.sum().backward()

    hr = h.detach().clone().requires_grad_()
    Wr = W.clone().requires_grad_()
    z = (hr @ Wr.t()) / tau
    for i, s in enumerate(supports):
        if s:
            blocked = torch.ones(V, dtype=torch.bool)
            blocked[s] = False
            z = z.masked_fill(torch.nn.functional.one_hot(torch.tensor(i), T).bool()[:, None] & blocked, float("-inf"))
    want = z.log_softmax(-1).gather(-1, tgt[:, None])[:, 0]
    want.sum().backward()
    torch.testing.assert_close(lp.detach(), want.detach(), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(h.grad, hr.grad, atol=1e-5, rtol=1e-5)
    # the full-vocabulary part of the head gradient flows through autograd of
    # the CPU reference only for row 2; the support rows land in gW
    full_rows = torch.zeros(V, H)
    z2 = (h.detach()[2:3] @ W.t()) / tau
    p = z2.softmax(-1)
    g = -p
    g[0, tgt[2]] += 1.0
    full_rows += (g / tau).t() @ h.detach()[2:3]
    torch.testing.assert_close(gW + full_rows, Wr.grad, atol=1e-5, rtol=1e-5)


def test_rows_without_support_use_full_vocabulary():
    torch.manual_seed(1)
    h, W = torch.randn(3, 4), torch.randn(6, 4)
    tgt = torch.tensor([0, 5, 2])
    lp = _support_lp(h, W, torch.zeros(6, 4), tgt, [[], [], []], 1.3)
    want = ((h @ W.t()) / 1.3).log_softmax(-1).gather(-1, tgt[:, None])[:, 0]
    torch.testing.assert_close(lp, want)
