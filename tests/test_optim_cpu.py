"""Non-AdamW optimizers over the flat store against per-tensor restatements of
the reference's rules (trainer/optim.py:30-188, 402-437): SGD against
``torch.optim.SGD`` itself, SignSGD and Muon against the formulas; Muon on 2
gloo ranks, with a matrix that straddles the shard boundary, matches one rank."""

import os
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from wavelet_b200.configs.config import OptimizerConfig
from wavelet_b200.models.params import FlatParams, ParamSpec
from wavelet_b200.trainer.optim import FlatOptimizer, newton_schulz5

SPECS = [
    ParamSpec("embed", (10, 8)),
    ParamSpec("layers.0.w", (40, 24)),  # elements 128..1088: crosses the 2-rank shard boundary at 704
    ParamSpec("layers.0.experts", (3, 4, 6)),
    ParamSpec("layers.0.norm", (8,), init="ones"),
    ParamSpec("lm_head", (10, 8)),
]
STEPS = 3


def _grads(step: int) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(100 + step)
    return {s.name: torch.randn(s.shape, generator=g) for s in SPECS}


def _run_flat(cfg: OptimizerConfig, rank: int = 0, world: int = 1, group=None) -> dict[str, torch.Tensor]:
    flat = FlatParams(SPECS, "cpu", torch.float32, rank, world)
    flat.init_(seed=3)
    flat.sync_master_from_compute()
    opt = FlatOptimizer(flat, cfg, max_grad_norm=0.0, dp_group=group, dp_world=world)
    for step in range(STEPS):
        for n, g in _grads(step).items():
            flat.grad_view(n).copy_(g / world)  # the reduce-scatter sums the ranks
        opt.step(cfg.lr)
    return {n: flat.view(n).clone() for n in flat.names()}


def _initial() -> dict[str, torch.Tensor]:
    flat = FlatParams(SPECS, "cpu", torch.float32)
    flat.init_(seed=3)
    return {n: flat.view(n).clone() for n in flat.names()}


def _ref_muon(cfg: OptimizerConfig) -> dict[str, torch.Tensor]:
    p = _initial()
    mom = {n: torch.zeros_like(t) for n, t in p.items()}
    m = {n: torch.zeros_like(t) for n, t in p.items()}
    v = {n: torch.zeros_like(t) for n, t in p.items()}
    beta, lr, wd = cfg.muon_momentum, cfg.lr, cfg.weight_decay
    b1, b2 = cfg.betas1, cfg.betas2
    for step in range(STEPS):
        for n, g in _grads(step).items():
            if g.dim() >= 2 and "embed" not in n and "lm_head" not in n:
                mom[n] = beta * mom[n] + (1 - beta) * g
                src = g + beta * mom[n] if cfg.nesterov else mom[n]
                upd = newton_schulz5(src)
                upd = upd * (g.norm() / upd.norm().clamp_min(1e-7))
            else:
                t = step + 1
                m[n] = b1 * m[n] + (1 - b1) * g
                v[n] = b2 * v[n] + (1 - b2) * g * g
                upd = (m[n] / (1 - b1**t)) / ((v[n] / (1 - b2**t)).sqrt() + 1e-8)
            p[n] = p[n] * (1 - lr * wd) - lr * upd
    return p


def test_newton_schulz_is_near_orthogonal_and_batched():
    x = torch.randn(2, 16, 48, generator=torch.Generator().manual_seed(0))
    o = newton_schulz5(x)
    assert o.shape == x.shape
    sv = torch.linalg.svdvals(o)
    assert float(sv.min()) > 0.5 and float(sv.max()) < 1.3  # the quintic's band around 1
    torch.testing.assert_close(o[1], newton_schulz5(x[1]))
    tall = newton_schulz5(x[0].t())
    torch.testing.assert_close(tall, o[0].t())


@pytest.mark.parametrize("nesterov", [True, False])
def test_muon_matches_reference_rule(nesterov):
    cfg = OptimizerConfig(type="muon", lr=0.02, weight_decay=0.1, nesterov=nesterov)
    got, ref = _run_flat(cfg), _ref_muon(cfg)
    for n in ref:
        torch.testing.assert_close(got[n], ref[n], rtol=1e-4, atol=1e-5, msg=n)
    assert not torch.equal(got["layers.0.w"], _initial()["layers.0.w"])


@pytest.mark.parametrize("nesterov", [True, False])
def test_sgd_matches_torch_sgd(nesterov):
    cfg = OptimizerConfig(type="sgd", lr=0.05, weight_decay=0.01, momentum=0.9, nesterov=nesterov)
    got = _run_flat(cfg)
    params = {n: torch.nn.Parameter(t) for n, t in _initial().items()}
    opt = torch.optim.SGD(params.values(), lr=cfg.lr, momentum=cfg.momentum, weight_decay=cfg.weight_decay,
                          nesterov=nesterov)
    for step in range(STEPS):
        for n, g in _grads(step).items():
            params[n].grad = g.clone()
        opt.step()
    for n, p in params.items():
        torch.testing.assert_close(got[n], p.detach(), rtol=1e-5, atol=1e-6, msg=n)


def test_sign_sgd_rule():
    cfg = OptimizerConfig(type="sign_sgd", lr=0.01, weight_decay=0.1)
    got, p = _run_flat(cfg), _initial()
    for step in range(STEPS):
        for n, g in _grads(step).items():
            p[n] = p[n] * (1 - cfg.lr * cfg.weight_decay) - cfg.lr * g.sign()
    for n in p:
        torch.testing.assert_close(got[n], p[n], rtol=1e-5, atol=1e-6, msg=n)


def _muon_worker(rank, world, init_file, out):
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    cfg = OptimizerConfig(type="muon", lr=0.02, weight_decay=0.1)
    res = _run_flat(cfg, rank, world, dist.group.WORLD)
    torch.save(res, f"{out}.{rank}")
    dist.destroy_process_group()


def test_muon_two_ranks_match_one():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_muon_worker, args=(world, os.path.join(d, "init"), os.path.join(d, "res")), nprocs=world, join=True)
        got = [torch.load(os.path.join(d, f"res.{r}")) for r in range(world)]
    ref = _run_flat(OptimizerConfig(type="muon", lr=0.02, weight_decay=0.1))
    for r in range(world):
        for n in ref:
            torch.testing.assert_close(got[r][n], ref[n], rtol=1e-5, atol=1e-6, msg=f"rank {r} {n}")


@pytest.mark.parametrize("kind", ["adamw", "sgd", "muon"])
def test_finite_gradients_with_overflowing_norm_abort_before_update(kind):
    from wavelet_b200.parallel.zero import NonFiniteGradientError

    flat = FlatParams(SPECS, "cpu", torch.float32)
    flat.init_(seed=3)
    flat.sync_master_from_compute()
    before = flat.master.clone()
    opt = FlatOptimizer(flat, OptimizerConfig(type=kind, lr=0.1), max_grad_norm=1.0)
    flat.grad.fill_(1e30)  # every element finite; the squared norm is not
    with pytest.raises(NonFiniteGradientError, match="overflows"):
        opt.step(0.1)
    assert torch.equal(flat.master, before)
    assert opt.step_count == 0


@pytest.mark.parametrize("kind", ["adamw", "sgd"])
def test_overflowing_norm_steps_when_clipping_is_off(kind):
    """With max_grad_norm = 0 the norm is not used, so finite gradients whose
    squared norm overflows still update (the reference checks it only when
    clipping)."""
    flat = FlatParams(SPECS, "cpu", torch.float32)
    flat.init_(seed=3)
    flat.sync_master_from_compute()
    before = flat.master.clone()
    opt = FlatOptimizer(flat, OptimizerConfig(type=kind, lr=0.1), max_grad_norm=0.0)
    flat.grad.fill_(1e18)  # each square is finite in fp32, their sum is not
    out = opt.step(0.1)
    assert out["clip_factor"] == 1.0
    assert torch.isfinite(flat.master).all()
    assert not torch.equal(flat.master, before)
    assert opt.step_count == 1


def test_non_finite_element_message_counts_elements():
    from wavelet_b200.parallel.zero import NonFiniteGradientError

    flat = FlatParams(SPECS, "cpu", torch.float32)
    flat.init_(seed=3)
    opt = FlatOptimizer(flat, OptimizerConfig(type="adamw", lr=0.1), max_grad_norm=0.0)
    flat.grad.zero_()
    flat.grad[5] = float("nan")
    flat.grad[9] = float("inf")
    with pytest.raises(NonFiniteGradientError, match=r"\(2 elements\)"):
        opt.step(0.1)
