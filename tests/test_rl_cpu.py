"""RL pieces on CPU: losses, algorithms, rewards, queue lifecycle, packing and
the integrated RL loop."""

import json
import math
import os
import subprocess
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

from wavelet_b200.configs.config import RLConfig, RLLossConfig, RLTransportConfig
from wavelet_b200.data.rl import RLExample, distribute_bins, make_rank_batches, pack_ffd, sample_from_example
from wavelet_b200.orchestrator.algorithms import GRPOAlgorithm, MaxRLAlgorithm, build_algorithm, group_reward_advantages
from wavelet_b200.orchestrator.reward import RLRewardScorer, reverse_match_score
from wavelet_b200.trainer.losses import compute_loss, dppo_loss, LossInputs
from wavelet_b200.transport.queue import FileSystemRolloutReceiver, FileSystemRolloutSender, read_training_records, scan_queue

ROOT = Path(__file__).resolve().parents[1]


def _span_reference(lp, ilp, adv, mask, cu, cfg):
    """Per-sequence loop formulation (what the vectorised version must equal)."""
    total = 0.0
    n_tok = 0
    for s, e in zip(cu[:-1].tolist(), cu[1:].tolist()):
        m = mask[s:e]
        if not m.any():
            continue
        out = dppo_loss(LossInputs(lp[s:e], ilp[s:e], None, adv[s:e], m), cfg)
        total = total + out.loss.sum()
        n_tok += int(m.sum())
    return total / max(n_tok, 1)


def test_dppo_loss_vectorised_matches_span_loop():
    torch.manual_seed(0)
    T = 50
    cu = torch.tensor([0, 10, 30, 50])
    lp = (torch.randn(T) * 0.5 - 1).requires_grad_(True)
    ilp = lp.detach() + 0.3 * torch.randn(T)
    adv = torch.randn(T)
    mask = torch.rand(T) > 0.3
    cfg = RLLossConfig()
    loss, met = compute_loss(lp, ilp, None, adv, mask, cfg, cu_seqlens=cu)
    ref = _span_reference(lp, ilp, adv, mask, cu, cfg)
    assert torch.allclose(loss, ref, atol=1e-6)
    assert "is_masked" in met and "mismatch_kl/median" in met


def test_sequence_normalisation():
    T = 6
    cu = torch.tensor([0, 2, 6])
    lp = torch.zeros(T, requires_grad=True)
    ilp = torch.zeros(T)
    adv = torch.ones(T)
    mask = torch.ones(T, dtype=torch.bool)
    cfg = RLLossConfig(normalization="sequence", kl_tau=0.0)
    loss, _ = compute_loss(lp, ilp, None, adv, mask, cfg, cu_seqlens=cu)
    # every token contributes -adv*ratio = -1; per-sequence means are -1; mean over 2 sequences
    assert abs(loss.item() - (-1.0)) < 1e-6


def test_grpo_and_maxrl():
    recs = [RLExample([], [], None, r) for r in (1.0, 0.0, 0.5, 0.5)]
    out = GRPOAlgorithm(normalize_advantages=False).score_group(recs)
    assert [round(r.advantage, 4) for r in out] == [0.5, -0.5, 0.0, 0.0]
    out = GRPOAlgorithm(normalize_advantages=True).score_group(recs)
    std = math.sqrt((0.25 + 0.25) / 4)
    assert abs(out[0].advantage - 0.5 / std) < 1e-6
    out = MaxRLAlgorithm().score_group(recs)
    assert abs(out[0].advantage - 1.0) < 1e-6
    assert group_reward_advantages([]) == []


def test_reverse_match_reward():
    assert reverse_match_score([1, 2, 3], [3, 2, 9, 9]) == 0.5
    cfg = RLConfig.model_validate({"reward": {"mode": "reverse_match"}}).reward
    r = RLExample([], [], None, None, input_ids=[1, 2, 3, 3, 2, 1], loss_mask=[False] * 3 + [True] * 3)
    assert RLRewardScorer(cfg).score(r) == 1.0


def test_queue_lifecycle(tmp_path):
    cfg = RLTransportConfig(poll_interval_seconds=0.01, idle_timeout_seconds=1.0, keep_last_consumed=1)
    s = FileSystemRolloutSender(tmp_path, cfg)
    rows = [{"prompt": [], "completion": [], "advantage": 1.0, "reward": 1.0, "input_ids": [1, 2, 3], "loss_mask": [False, True, True]}]
    s.publish(rows, step=0, training_records=rows)
    s.publish(rows, step=1, training_records=rows)
    with pytest.raises(FileExistsError):
        s.publish(rows, step=1)
    r = FileSystemRolloutReceiver(tmp_path, cfg)
    b = r.wait()
    assert b.step == 0 and b.training_path.name.endswith(".train.msgpack")
    assert read_training_records(b.training_path)[0]["input_ids"] == [1, 2, 3]
    r.claim(b, 0)
    r.consumed(b, 0, 1)
    b1 = r.wait()
    r.consumed(b1, 1, 2)
    st = scan_queue(s.queue_dir)
    assert st["counts"] == {"consumed": 1}
    with pytest.raises(TimeoutError):
        r.wait()
    ev = [json.loads(l)["kind"] for l in (tmp_path / "events" / "queue.jsonl").read_text().splitlines()]
    assert ev.count("rollout_published") == 2 and "rollout_consumed" in ev


def test_alignment_and_packing():
    e = RLExample([], [], 2.0, 1.0, input_ids=[5, 6, 7, 8], loss_mask=[False, False, True, True],
                  inference_logprobs=[-0.5, -0.25])
    s = sample_from_example(e)
    assert s.loss_mask.tolist() == [False, True, True, False]
    assert s.inference_logprobs.tolist() == [0.0, -0.5, -0.25, 0.0]
    assert s.advantages.tolist() == [0.0, 2.0, 2.0, 0.0]
    bins = pack_ffd([5, 3, 4, 2, 6], 8)
    assert sorted(sum(bins, [])) == [0, 1, 2, 3, 4] and all(sum([5, 3, 4, 2, 6][i] for i in b) <= 8 for b in bins)
    per = distribute_bins(bins, [5, 3, 4, 2, 6], 2)
    assert len(per[0]) == len(per[1])
    exs = [RLExample([], [], 1.0, 1.0, input_ids=list(range(10)), loss_mask=[False] * 5 + [True] * 5)] * 6
    b0 = make_rank_batches(exs, 32, 0, 2)
    b1 = make_rank_batches(exs, 32, 1, 2)
    assert len(b0) == len(b1)


@pytest.mark.integration
def test_integrated_rl_cpu(tmp_path):
    cfg = tmp_path / "rl.yaml"
    cfg.write_text(
        f"""model:
  name: tiny
  random_init: true
data:
  source: fake
  seq_len: 128
  fake_vocab_size: 64
  fake_prompt_len: 8
algo:
  type: grpo
reward:
  mode: reverse_match
orchestrator:
  examples_per_step: 4
  rollouts_per_example: 4
inference:
  sampling:
    max_completion_tokens: 8
lora: null
max_steps: 3
output_dir: {tmp_path / 'out'}
"""
    )
    env = {**os.environ, "WAVELET_FORCE_CPU": "1"}
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "rl", "@", str(cfg)], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    rows = [json.loads(l) for l in (tmp_path / "out" / "metrics.jsonl").read_text().splitlines()]
    assert [x["step"] for x in rows] == [1, 2, 3]
    assert "reward/mean" in rows[0] and "rollout/tokens_per_second" in rows[0]


def test_mixed_sampling_temperatures_pack_apart():
    exs = [RLExample([], [], 1.0, 1.0, input_ids=list(range(6)), loss_mask=[False] * 3 + [True] * 3,
                     temperatures=t) for t in (0.7, 1.0, 0.7, 1.0, 1.0)]
    batches = make_rank_batches(exs, 64, 0, 1)
    temps = sorted(b.temperature for b in batches if b.num_samples)
    assert temps == [0.7, 1.0]  # one bin per temperature, no mixing
    assert sum(b.num_samples for b in batches) == 5
