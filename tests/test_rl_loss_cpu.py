"""RL losses on the packed layout against the values the reference's loss
tests pin (tests/test_rl_loss.py of the reference): trust-region overflow,
IcePop bands, token / sequence normalisation, IPO masks, per-sequence
metrics, the DPPO golden loss, CE / ref-KL component scales, unit counts and
the per-span custom-loss contract."""

import math
import sys
import types

import pytest
import torch

from wavelet_b200.configs.config import RLLossConfig
from wavelet_b200.trainer.losses import LossInputs, LossOutput, component_unit_counts, compute_loss, segment_ids


def _cu(position_ids, T):
    if position_ids is None:
        return torch.tensor([0, T])
    starts = (position_ids.reshape(-1) == 0).nonzero().flatten().tolist()
    if not starts or starts[0] != 0:
        starts = [0, *starts]
    return torch.tensor([*starts, T])


def _loss(trainer, inference, teacher, adv, mask, cfg, *, loss_scale=None, position_ids=None,
          component_loss_scales=None, **weights):
    """The reference's [1, T] call shape mapped onto the packed [T] API."""
    T = trainer.shape[-1]
    flat = lambda t: None if t is None else t.reshape(-1)  # noqa: E731
    scales = dict(component_loss_scales or {})
    if loss_scale is not None and "rl" not in scales:
        scales["rl"] = loss_scale
    return compute_loss(flat(trainer), flat(inference), flat(teacher), flat(adv), flat(mask), cfg,
                        cu_seqlens=_cu(position_ids, T), component_scales=scales or None,
                        **{k: flat(v) for k, v in weights.items()})


@pytest.mark.parametrize("loss_type", ["dppo", "ipo"])
def test_trust_region_rejects_overflowing_ratios_before_exp(loss_type):
    trainer = torch.tensor([[-1.0, -1.0]], requires_grad=True)
    loss, m = _loss(trainer, torch.full((1, 2), -100.0), None, torch.ones(1, 2), torch.tensor([[True, False]]),
                    RLLossConfig(type=loss_type, kl_tau=0.01))
    loss.backward()
    assert loss.item() == pytest.approx(0.01 * 99**2)
    torch.testing.assert_close(trainer.grad, torch.tensor([[1.98, 0.0]]))
    assert m["is_masked"] == 1.0


def test_ref_kl_ignores_overflowing_ratios_outside_component_mask():
    trainer = torch.tensor([[-1.0, -1.0]], requires_grad=True)
    loss, _ = _loss(trainer, torch.tensor([[-1.0, -100.0]]), torch.full((1, 2), -2.0), torch.zeros(1, 2),
                    torch.ones(1, 2, dtype=torch.bool), RLLossConfig(), rl_weights=torch.zeros(1, 2),
                    ref_kl_weights=torch.tensor([[1.0, 0.0]]))
    loss.backward()
    assert torch.isfinite(loss)
    torch.testing.assert_close(trainer.grad, torch.tensor([[1.0, 0.0]]))


def test_icepop_masks_out_of_band_ratios_without_nan():
    trainer = torch.tensor([0.1, 0.2, 1.0, 5.0, 10.0]).log().unsqueeze(0).requires_grad_()
    loss, m = _loss(trainer, torch.zeros(1, 5), None, torch.ones(1, 5), torch.ones(1, 5, dtype=torch.bool),
                    RLLossConfig(type="icepop", ratio_low=0.2, ratio_high=5.0), loss_scale=1)
    assert m["is_masked"] == pytest.approx(0.4)
    loss.backward()
    assert torch.isfinite(trainer.grad).all()


def test_token_and_sequence_normalisation():
    adv = torch.tensor([[2.0, 2.0, 2.0, -1.0]])
    pos = torch.tensor([[0, 1, 2, 0]])
    z = torch.zeros(1, 4)
    ones = torch.ones(1, 4, dtype=torch.bool)
    tok, _ = _loss(z, z, None, adv, ones, RLLossConfig(kl_tau=0.0), loss_scale=4, position_ids=pos)
    assert tok.item() == pytest.approx(-1.25)
    seq, _ = _loss(z, z, None, adv, ones, RLLossConfig(kl_tau=0.0, normalization="sequence"), loss_scale=2,
                   position_ids=pos)
    assert seq.item() == pytest.approx(-0.5)


def test_unit_counts_follow_packed_boundaries():
    mask = torch.tensor([True, True, False, True, False])
    seg = segment_ids(_cu(torch.tensor([0, 1, 2, 0, 1]), 5), 5)
    assert component_unit_counts(mask, seg, 2, rl_normalization="token")["rl"] == 3
    assert component_unit_counts(mask, seg, 2, rl_normalization="sequence")["rl"] == 2
    seg = segment_ids(_cu(torch.tensor([0, 1, 0, 1]), 4), 4)
    counts = component_unit_counts(torch.ones(4, dtype=torch.bool), seg, 2,
                                   rl_weights=torch.tensor([1.0, 0.0, 0.0, 1.0]),
                                   ce_weights=torch.tensor([0.0, 2.0, 0.0, 0.0]),
                                   ref_kl_weights=torch.tensor([0.0, 0.0, -1.0, 1.0]), rl_normalization="sequence")
    assert counts == {"rl": 2, "ce": 1, "ref_kl": 2}


def test_policy_gradient_moves_logprobs_in_advantage_direction():
    lp = torch.zeros((1, 2), requires_grad=True)
    opt = torch.optim.SGD([lp], lr=0.1)
    loss, _ = _loss(lp, torch.zeros(1, 2), None, torch.tensor([[1.0, -1.0]]), torch.ones(1, 2, dtype=torch.bool),
                    RLLossConfig(kl_tau=0.0), loss_scale=2)
    loss.backward()
    opt.step()
    assert lp[0, 0].item() > 0.0 and lp[0, 1].item() < 0.0


def test_ipo_masks_probability_moves_symmetrically():
    lp = torch.log(torch.tensor([[0.32, 0.18, 0.59, 0.41]])).requires_grad_()
    loss, m = _loss(lp, torch.log(torch.tensor([[0.20, 0.30, 0.50, 0.50]])), None,
                    torch.tensor([[1.0, 1.0, 1.0, -1.0]]), torch.ones(1, 4, dtype=torch.bool),
                    RLLossConfig(type="ipo", ipo_epsilon=0.1, kl_tau=0.0), loss_scale=4)
    loss.backward()
    assert m["is_masked"] == pytest.approx(0.5)
    assert m["is_masked_high"] == pytest.approx(0.25) and m["is_masked_low"] == pytest.approx(0.25)
    torch.testing.assert_close(lp.grad[0, :2], torch.zeros(2))
    assert lp.grad[0, 2].item() < 0.0 and lp.grad[0, 3].item() > 0.0


def test_metrics_are_averaged_per_sequence():
    _, m = _loss(torch.tensor([[0.0, 0.0, 0.0, math.log(0.5)]]), torch.tensor([[0.0, 0.0, 0.0, math.log(0.25)]]),
                 None, torch.zeros(1, 4), torch.ones(1, 4, dtype=torch.bool), RLLossConfig(kl_tau=0.0), loss_scale=4,
                 position_ids=torch.tensor([[0, 1, 2, 0]]))
    assert m["mismatch_kl"] == pytest.approx((2.0 - math.log(2.0) - 1.0) / 2)


def test_dppo_golden_value_and_component_form():
    lp = torch.tensor([[math.log(0.3), math.log(0.7), math.log(0.2)]], requires_grad=True)
    inf = torch.tensor([[math.log(0.25), math.log(0.6), math.log(0.25)]])
    teacher = torch.tensor([[math.log(0.4), math.log(0.65), math.log(0.3)]])
    cfg = RLLossConfig(dppo_mask_high=0.2, dppo_mask_low=0.2, kl_tau=0.01, adv_tau=0.8, teacher_tau=0.15)
    adv = torch.tensor([[1.25, -0.5, 0.75]])
    mask = torch.ones(1, 3, dtype=torch.bool)
    legacy, lm = _loss(lp, inf, teacher, adv, mask, cfg, loss_scale=3)
    comp, cm = _loss(lp, inf, teacher, adv, mask, cfg, loss_scale=3, rl_weights=torch.ones(1, 3),
                     ce_weights=torch.zeros(1, 3), ref_kl_weights=torch.zeros(1, 3),
                     component_loss_scales={"rl": 3.0, "ce": 1.0, "ref_kl": 1.0})
    assert legacy.item() == pytest.approx(-0.43324506282806396)
    assert torch.equal(comp, legacy)
    assert cm == lm


def test_ce_and_ref_kl_use_independent_token_scales():
    lp = torch.full((1, 4), -1.0)
    loss, m = _loss(lp, lp.clone(), torch.tensor([[0.0, 1.0, 2.0, 3.0]]), torch.zeros(1, 4),
                    torch.ones(1, 4, dtype=torch.bool), RLLossConfig(), rl_weights=torch.zeros(1, 4),
                    ce_weights=torch.tensor([[0.0, 2.0, 1.0, 0.0]]), ref_kl_weights=torch.tensor([[1.0, 2.0, 0.0, 0.0]]),
                    component_loss_scales={"rl": 1.0, "ce": 2.0, "ref_kl": 2.0})
    assert loss.item() == pytest.approx(1.5 - 2.5)
    assert m["ce/nll"] == pytest.approx(1.0) and m["ref_kl"] == pytest.approx(1.5)


def test_component_metrics_skip_sequences_without_component_tokens():
    # two sequences; only the second has CE tokens: the CE metric is its mean alone
    lp = torch.tensor([-1.0, -1.0, -3.0, -5.0])
    _, m = compute_loss(lp, lp.clone(), None, torch.zeros(4), torch.ones(4, dtype=torch.bool), RLLossConfig(),
                        cu_seqlens=torch.tensor([0, 2, 4]), rl_weights=torch.zeros(4),
                        ce_weights=torch.tensor([0.0, 0.0, 1.0, 1.0]))
    assert m["ce/nll"] == pytest.approx(4.0) and m["ce/nll/min"] == pytest.approx(4.0)


def test_ref_kl_one_sided_trust_region_and_teacher_requirement():
    _, m = _loss(torch.tensor([[math.log(0.1), math.log(0.8)]]), torch.tensor([[math.log(0.5), math.log(0.5)]]),
                 torch.tensor([[math.log(0.9), math.log(0.9)]]), torch.zeros(1, 2), torch.ones(1, 2, dtype=torch.bool),
                 RLLossConfig(), rl_weights=torch.zeros(1, 2), ref_kl_weights=torch.ones(1, 2),
                 component_loss_scales={"rl": 1.0, "ce": 1.0, "ref_kl": 2.0})
    assert m["ref_kl/is_masked"] == pytest.approx(0.5)
    with pytest.raises(ValueError, match="requires teacher_logprobs"):
        _loss(torch.zeros(1, 1), torch.zeros(1, 1), None, torch.zeros(1, 1), torch.ones(1, 1, dtype=torch.bool),
              RLLossConfig(), rl_weights=torch.zeros(1, 1), ref_kl_weights=torch.ones(1, 1))


def test_custom_loss_is_imported_called_per_span_with_kwargs(monkeypatch):
    mod = types.ModuleType("wavelet_b200_test_custom_loss")
    calls = []

    def custom_loss(inputs: LossInputs, *, multiplier: float) -> LossOutput:
        calls.append(inputs.trainer_logprobs.numel())
        loss = -(inputs.trainer_logprobs[inputs.loss_mask] * multiplier).sum()
        return LossOutput(loss=loss, metrics={"custom": loss.detach()})

    mod.custom_loss = custom_loss
    monkeypatch.setitem(sys.modules, mod.__name__, mod)
    cfg = RLLossConfig(type="custom", import_path=f"{mod.__name__}.custom_loss", kwargs={"multiplier": 2.0})
    loss, m = _loss(torch.tensor([[-1.0, -2.0]]), torch.zeros(1, 2), None, torch.zeros(1, 2),
                    torch.ones(1, 2, dtype=torch.bool), cfg, loss_scale=2)
    assert loss.item() == pytest.approx(3.0) and m["custom"] == pytest.approx(6.0)
    calls.clear()
    loss, m = _loss(torch.tensor([[-1.0, -2.0, -3.0]]), torch.zeros(1, 3), None, torch.zeros(1, 3),
                    torch.ones(1, 3, dtype=torch.bool), cfg, loss_scale=1, position_ids=torch.tensor([[0, 1, 0]]))
    assert calls == [2, 1]  # one call per packed sequence
    assert loss.item() == pytest.approx(12.0) and m["custom"] == pytest.approx(6.0)
    assert m["custom/min"] == pytest.approx(6.0) and m["custom/max"] == pytest.approx(6.0)
