"""8-bit AdamW (block-scaled log-coded moments): code round trip, tracking of
fp32 AdamW on a least-squares problem, optimizer types wired to it, and the
checkpoint re-shard path through fp32 moments."""

import math

import pytest
import torch

from wavelet_b200 import ops
from wavelet_b200.configs.config import OptimizerConfig
from wavelet_b200.models.params import FlatParams, ParamSpec
from wavelet_b200.trainer.optim import FlatOptimizer


def test_log_codes_round_trip_within_one_step():
    torch.manual_seed(0)
    x = torch.randn(4096) * torch.exp2(torch.randint(-12, 3, (4096,)).float())
    a = x.abs().max()
    m = ops.q8m_decode(ops.q8m_encode(x, a), a)
    rel = ((m - x).abs() / x.abs().clamp_min(1e-30))
    big = x.abs() > a * 2.0 ** -14
    assert float(rel[big].max()) <= 2.0 ** (1 / 16) - 1 + 1e-6  # half a 2^(1/8) step
    assert torch.equal(torch.sign(m[big]), torch.sign(x[big]))
    v = x * x
    av = v.max()
    vv = ops.q8v_decode(ops.q8v_encode(v, av), av)
    relv = ((vv - v).abs() / v.clamp_min(1e-30))
    bigv = v > av * 2.0 ** -15
    assert float(relv[bigv].max()) <= 2.0 ** (1 / 32) - 1 + 1e-6
    assert ops.q8m_encode(torch.zeros(3), torch.tensor(1.0)).abs().sum() == 0


def _problem(seed=0):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(256, 64, generator=g)
    w_true = torch.randn(64, generator=g)
    b = A @ w_true
    return A, b


def _train(kind, steps=60):
    A, b = _problem()
    flat = FlatParams([ParamSpec("w", (64,), "zeros", True)], "cpu", torch.float32)
    flat.sync_master_from_compute()
    opt = FlatOptimizer(flat, OptimizerConfig(type=kind, lr=0.05, weight_decay=0.01), max_grad_norm=0.0)
    losses = []
    for _ in range(steps):
        w = flat.view("w").clone().requires_grad_(True)
        loss = ((A @ w - b) ** 2).mean()
        loss.backward()
        flat.grad_view("w").copy_(w.grad)
        losses.append(float(loss))
        opt.step(0.05)
    return losses, flat.master.clone()


@pytest.mark.parametrize("kind", ["adamw_8bit", "paged_adamw_8bit", "adam_8bit"])
def test_8bit_adamw_tracks_fp32_adamw(kind):
    ref_kind = "adam" if kind == "adam_8bit" else "adamw"
    l32, w32 = _train(ref_kind)
    l8, w8 = _train(kind)
    assert l8[-1] < 0.05 * l8[0]  # it optimises
    assert abs(l8[-1] - l32[-1]) <= 0.25 * l32[-1] + 1e-3
    assert float((w8 - w32).norm() / w32.norm()) < 0.05


def test_8bit_state_is_small_and_checkpoint_reshards_through_fp32():
    flat = FlatParams([ParamSpec("w", (1000,), "normal", True)], "cpu", torch.float32)
    flat.init_(seed=1)
    opt = FlatOptimizer(flat, OptimizerConfig(type="adamw_8bit", lr=0.1), max_grad_norm=1.0)
    assert flat.exp_avg is None and flat.exp_avg_sq is None
    for i in range(3):
        flat.grad.copy_(torch.randn(flat.numel) * (i + 1))
        opt.step(0.1)
    sd = opt.state_dict()
    assert sd["m8"].dtype == torch.int8 and sd["v8"].dtype == torch.uint8
    m, v = ops.q8_dequant_moments(sd["m8"], sd["v8"], sd["m8_scale"], sd["v8_scale"])
    flat2 = FlatParams([ParamSpec("w", (1000,), "normal", True)], "cpu", torch.float32)
    opt2 = FlatOptimizer(flat2, OptimizerConfig(type="adamw_8bit", lr=0.1), max_grad_norm=1.0)
    opt2.load_state_dict({"step": sd["step"], "master": sd["master"], "exp_avg": m, "exp_avg_sq": v})
    m2, v2 = ops.q8_dequant_moments(opt2.adamw.m8, opt2.adamw.v8, opt2.adamw.am, opt2.adamw.av)
    torch.testing.assert_close(m2, m, rtol=0.07, atol=1e-12)
    torch.testing.assert_close(v2, v, rtol=0.05, atol=1e-12)
    assert opt2.step_count == 3
