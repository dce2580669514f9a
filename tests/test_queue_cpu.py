"""Rollout queue behaviour the reference's queue tests pin (tests/test_queue.py
of the reference): out-of-order publication, late gaps, STABLE only after the
manifest, no overwrite of a stable batch, manifest and event contents, the
binary training sidecar and its JSON fallback."""

import json

import pytest

from wavelet_b200.configs.config import RLTransportConfig
from wavelet_b200.transport import queue as q
from wavelet_b200.transport.queue import FileSystemRolloutReceiver, FileSystemRolloutSender, read_training_records

CFG = RLTransportConfig(poll_interval_seconds=0.001, idle_timeout_seconds=2.0)
ROWS = [{"value": 1}]


def test_wait_available_takes_oldest_and_skips_missing_step(tmp_path):
    s = FileSystemRolloutSender(tmp_path, CFG)
    s.publish(ROWS, step=2)
    s.publish(ROWS, step=1)
    r = FileSystemRolloutReceiver(tmp_path, CFG)
    assert r.wait_available().step == 1
    assert r.wait_available().step == 2


def test_wait_available_picks_up_a_late_gap(tmp_path):
    s = FileSystemRolloutSender(tmp_path, CFG)
    s.publish(ROWS, step=1)
    r = FileSystemRolloutReceiver(tmp_path, CFG)
    assert r.wait_available().step == 1
    s.publish(ROWS, step=0)
    assert r.wait_available().step == 0
    assert r.next_step == 2
    with pytest.raises(TimeoutError):
        FileSystemRolloutReceiver(tmp_path, RLTransportConfig(poll_interval_seconds=0.001, idle_timeout_seconds=0.05),
                                  start_step=2).wait_available()


def test_manifest_failure_leaves_batch_unstable(tmp_path, monkeypatch):
    s = FileSystemRolloutSender(tmp_path, CFG)

    def fail(*_a, **_k):
        raise OSError("disk full")

    monkeypatch.setattr(q, "_write_json", fail)
    with pytest.raises(OSError, match="disk full"):
        s.publish(ROWS, step=0, optimizer_step=0)
    assert not (q.step_dir(s.queue_dir, 0) / q.STABLE).exists()
    assert s.stable_batch(0) is None


def test_stable_batch_cannot_be_overwritten(tmp_path):
    s = FileSystemRolloutSender(tmp_path, CFG)
    b = s.publish([{"value": 1}], step=0)
    with pytest.raises(FileExistsError, match="already stable"):
        s.publish([{"value": 2}], step=0)
    assert s.stable_batch(0) == b
    assert b.path.read_text() == '{"value": 1}\n'


def test_manifest_and_event_contents(tmp_path):
    s = FileSystemRolloutSender(tmp_path, CFG)
    b = s.publish(ROWS, step=0, optimizer_step=0, policy_step=0, tokens=5, reward_mean=0.5)
    m = b.manifest
    assert (m.queue_step, m.optimizer_step, m.policy_step, m.rows, m.tokens) == (0, 0, 0, 1, 5)
    assert m.payload_bytes == len('{"value": 1}\n') and m.transfer_seconds >= 0
    ev = json.loads((tmp_path / "events" / "queue.jsonl").read_text().splitlines()[-1])
    assert ev["kind"] == "rollout_published" and ev["details"]["payload_bytes"] == m.payload_bytes


def test_binary_sidecar_and_json_fallback(tmp_path):
    s = FileSystemRolloutSender(tmp_path, CFG)
    rec = [{"input_ids": [1, 2, 3], "trace": {"tool": "x"}}]
    b = s.publish(rec, step=0, training_records=rec)
    assert b.training_path.name.endswith(q.TRAIN_SUFFIX)
    assert read_training_records(b.training_path) == rec
    huge = [{"input_ids": [1], "metadata": {"id": 1 << 70}}]  # beyond msgpack's 64-bit integers
    b = s.publish(huge, step=1, training_records=huge)
    assert b.training_path == b.path  # no sidecar: the JSON rows are the training records
    assert read_training_records(b.training_path)[0]["metadata"]["id"] == 1 << 70
