"""Rollout queue and policy snapshot lifecycle on the filesystem (ref
transport/queue.py; behaviours of the reference's queue-lifecycle and
artifact-retention tests): manifests, claim / consumed records, events,
pruning, resume discards and snapshot retention."""

from __future__ import annotations

import json

import pytest

from wavelet_b200.configs.config import RLConfig
from wavelet_b200.transport.queue import (CLAIM, CONSUMED, STABLE, FileSystemPolicyReceiver,
                                          FileSystemRolloutReceiver, FileSystemRolloutSender, prune_consumed,
                                          prune_from, read_training_records, scan_queue, stable_steps, step_dir)


def _cfg(tmp_path, **transport):
    return RLConfig.model_validate({"output_dir": str(tmp_path / "out"),
                                    "transport": {"poll_interval_seconds": 0.01, "idle_timeout_seconds": 1.0,
                                                  **transport},
                                    "policy_transfer": {"poll_interval_seconds": 0.01, "idle_timeout_seconds": 1.0}})


def _rows(n, step):
    return [{"prompt": [], "completion": [], "advantage": 0.5, "reward": 1.0, "input_ids": [step, i],
             "loss_mask": [False, True]} for i in range(n)]


def test_manifest_claim_and_consumed_round_trip(tmp_path):
    cfg = _cfg(tmp_path)
    out = tmp_path / "out"
    s = FileSystemRolloutSender(out, cfg.transport)
    b = s.publish(_rows(3, 0), step=0, training_records=_rows(3, 0), optimizer_step=0, policy_step=0, tokens=6,
                  reward_mean=1.0, prompt_source_state={"cursor": 3})
    man = b.manifest
    assert (man.queue_step, man.rows, man.tokens, man.policy_step) == (0, 3, 6, 0)
    assert man.prompt_source_state == {"cursor": 3} and man.payload_bytes > 0 and man.producer_id
    assert read_training_records(b.training_path)[2]["input_ids"] == [0, 2]  # the msgpack sidecar
    with pytest.raises(FileExistsError, match="already stable"):
        s.publish(_rows(1, 0), step=0)
    r = FileSystemRolloutReceiver(out, cfg.transport, consumer_id="trainer-a")
    got = r.wait()
    r.claim(got, 0)
    claim = json.loads((got.step_dir / CLAIM).read_text())
    assert claim["consumer_id"] == "trainer-a" and claim["trainer_step_before"] == 0
    r.consumed(got, 0, 1)
    done = json.loads((got.step_dir / CONSUMED).read_text())
    assert done["trainer_step_after"] == 1 and done["optimizer_step_completed"] is True
    kinds = [json.loads(l)["kind"] if "kind" in json.loads(l) else json.loads(l).get("event")
             for f in (out / "events").rglob("*.jsonl") for l in f.read_text().splitlines()]
    assert {"rollout_published", "rollout_received", "rollout_claimed", "rollout_consumed"} <= set(kinds)
    assert scan_queue(s.queue_dir)["counts"] == {"consumed": 1}


def test_receiver_waits_in_order_and_times_out(tmp_path):
    cfg = _cfg(tmp_path)
    out = tmp_path / "out"
    s = FileSystemRolloutSender(out, cfg.transport)
    s.publish(_rows(1, 1), step=1)
    r = FileSystemRolloutReceiver(out, cfg.transport)
    with pytest.raises(TimeoutError):
        r.wait()  # step 0 never appears
    a = FileSystemRolloutReceiver(out, cfg.transport)
    assert a.wait_available().step == 1  # any unconsumed batch
    s.publish(_rows(1, 0), step=0)
    assert a.wait_available().step == 0 and a.next_step == 2  # a late lower step is still taken
    with pytest.raises(TimeoutError):
        a.wait_available()


def test_pruning_keeps_recent_consumed_batches_and_resume_discards(tmp_path):
    cfg = _cfg(tmp_path, cleanup_consumed=False)
    out = tmp_path / "out"
    s = FileSystemRolloutSender(out, cfg.transport)
    r = FileSystemRolloutReceiver(out, cfg.transport)
    for step in range(5):
        s.publish(_rows(1, step), step=step)
    for step in range(4):
        b = r.wait()
        r.consumed(b, step, step + 1)
    assert prune_consumed(s.queue_dir, keep_last=2) == [0, 1]
    assert stable_steps(s.queue_dir) == [2, 3, 4]  # unconsumed step 4 is never pruned
    assert prune_from(s.queue_dir, 3) == [3, 4]
    assert stable_steps(s.queue_dir) == [2]
    # an unfinished (not STABLE) step directory is invisible to receivers
    step_dir(s.queue_dir, 7).mkdir(parents=True)
    assert 7 not in stable_steps(s.queue_dir)
    assert scan_queue(s.queue_dir)["counts"] == {"consumed": 1, "writing": 1}


def test_cleanup_consumed_prunes_on_consume(tmp_path):
    cfg = _cfg(tmp_path, cleanup_consumed=True, keep_last_consumed=1)
    out = tmp_path / "out"
    s = FileSystemRolloutSender(out, cfg.transport)
    r = FileSystemRolloutReceiver(out, cfg.transport)
    for step in range(3):
        s.publish(_rows(1, step), step=step)
        r.consumed(r.wait(), step, step + 1)
    assert stable_steps(s.queue_dir) == [2]


def test_policy_snapshots_export_once_and_keep_the_latest(tmp_path):
    import torch

    from wavelet_b200.models.config import resolve_arch
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.transport.policy import PolicyExporter

    cfg = RLConfig.model_validate({"output_dir": str(tmp_path / "out"),
                                   "policy_transfer": {"keep_last": 2, "poll_interval_seconds": 0.01,
                                                       "idle_timeout_seconds": 1.0}})
    model = build_model(resolve_arch("tiny"), torch.device("cpu"), seed=0, with_grad=False, with_optimizer=False)
    ex = PolicyExporter(tmp_path / "out", cfg.policy_transfer)
    d0 = ex.export(model, 0)
    meta = json.loads((d0 / "policy.json").read_text())
    assert meta["step"] == 0 and meta["kind"] == "model" and (d0 / STABLE).exists()
    stamp = (d0 / "policy.json").stat().st_mtime_ns
    assert ex.export(model, 0) == d0 and (d0 / "policy.json").stat().st_mtime_ns == stamp  # stable: not rewritten
    for s in (1, 2, 3):
        ex.export(model, s)
    assert stable_steps(ex.policy_dir) == [2, 3]  # keep_last
    rec = FileSystemPolicyReceiver(tmp_path / "out", cfg.policy_transfer)
    assert rec.wait_for_step(1).step == 3  # a pruned step is served by the newest snapshot
    assert rec.latest().step == 3
    with pytest.raises(TimeoutError):
        rec.wait_for_step(9)
