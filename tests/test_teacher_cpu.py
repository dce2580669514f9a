"""Distillation teacher log-probs: OPD scores rollouts on a teacher server's
/score route, OPSD on the policy itself behind a demonstration turn; the
log-probs land one per trainable token, equal to the teacher's
teacher-forced log-probs; other algorithms are untouched; integrated OPD
training against a running teacher server."""

import json
import os
import socket
import subprocess
import sys
import time
import urllib.request
from pathlib import Path

import pytest
import torch

from wavelet_b200.configs.config import RLConfig
from wavelet_b200.data.rl import RLExample
from wavelet_b200.models.config import PRESETS
from wavelet_b200.models.qwen import build_model
from wavelet_b200.orchestrator.teacher import attach_teacher_logprobs, model_scorer, opsd_prefix

ROOT = Path(__file__).resolve().parents[1]


def _rec(ids, n_prompt, **md):
    return RLExample(prompt=[], completion=[], advantage=0.0, reward=0.0, input_ids=ids,
                     loss_mask=[False] * n_prompt + [True] * (len(ids) - n_prompt), metadata=md)


def _want(model, seq, positions):
    with torch.no_grad():
        z = model.logits(model.hidden(torch.tensor(seq), model.batch_ctx(
            torch.arange(len(seq), dtype=torch.int32), torch.tensor([0, len(seq)], dtype=torch.int32), len(seq))))
        lp = torch.log_softmax(z.float(), -1)
    return [float(lp[j - 1, seq[j]]) for j in positions]


def test_opd_and_opsd_alignment():
    teacher = build_model(PRESETS["tiny"], "cpu", torch.float32, seed=4)
    recs = [_rec([5, 9, 13, 2, 7, 8], 3, demonstration="abc"), _rec([3, 3, 8, 1], 2, demonstration="xyz")]
    cfg = RLConfig.model_validate({"algo": {"type": "opd", "teacher": {"name": "t", "base_url": "http://x"}}})
    out = attach_teacher_logprobs(recs, cfg, scorer=model_scorer(teacher))
    for r, o in zip(recs, out):
        pos = [i for i, m in enumerate(r.loss_mask) if m]
        assert len(o.teacher_logprobs) == len(pos)
        torch.testing.assert_close(torch.tensor(o.teacher_logprobs), torch.tensor(_want(teacher, r.input_ids, pos)),
                                   rtol=1e-5, atol=1e-5)
    from wavelet_b200.data.tokenizer import CharTokenizer

    tok = CharTokenizer()
    cfg = RLConfig.model_validate({"algo": {"type": "opsd"}})
    out = attach_teacher_logprobs(recs, cfg, scorer=model_scorer(teacher), tokenizer=tok)
    pre = opsd_prefix(recs[0], cfg.algo, tok)
    assert len(pre) > 0
    pos = [i for i, m in enumerate(recs[0].loss_mask) if m]
    want = _want(teacher, pre + recs[0].input_ids, [len(pre) + i for i in pos])
    torch.testing.assert_close(torch.tensor(out[0].teacher_logprobs), torch.tensor(want), rtol=1e-5, atol=1e-5)
    with pytest.raises(ValueError, match="demonstration"):
        attach_teacher_logprobs([_rec([1, 2, 3], 1)], cfg, scorer=model_scorer(teacher), tokenizer=tok)
    grpo = RLConfig.model_validate({"algo": {"type": "grpo"}})
    assert attach_teacher_logprobs(recs, grpo)[0].teacher_logprobs is None


def _free():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.integration
def test_integrated_opd_against_a_teacher_server(tmp_path):
    env = {**os.environ, "WAVELET_FORCE_CPU": "1", "CUDA_VISIBLE_DEVICES": ""}
    port = _free()
    tcfg = tmp_path / "teacher.yaml"
    tcfg.write_text(f"""model:
  name: tiny
  random_init: true
seed: 9
data:
  source: fake
  seq_len: 128
inference:
  http:
    port: {port}
lora: null
output_dir: {tmp_path / 'teacher'}
""")
    srv = subprocess.Popen([sys.executable, "-m", "wavelet_b200", "inference-server", "@", str(tcfg)], cwd=ROOT,
                           env=env, stdout=subprocess.DEVNULL, stderr=subprocess.PIPE, start_new_session=True)
    try:
        t0 = time.monotonic()
        while True:
            try:
                urllib.request.urlopen(f"http://127.0.0.1:{port}/health", timeout=2)
                break
            except OSError:
                assert srv.poll() is None and time.monotonic() - t0 < 120
                time.sleep(0.5)
        cfg = tmp_path / "rl.yaml"
        cfg.write_text(f"""model:
  name: tiny
  random_init: true
data:
  source: fake
  seq_len: 128
  fake_vocab_size: 64
  fake_prompt_len: 8
algo:
  type: opd
  teacher:
    name: tiny
    base_url: http://127.0.0.1:{port}/v1
reward:
  mode: reverse_match
orchestrator:
  examples_per_step: 2
  rollouts_per_example: 2
inference:
  sampling:
    max_completion_tokens: 6
lora: null
max_steps: 2
output_dir: {tmp_path / 'out'}
""")
        r = subprocess.run([sys.executable, "-m", "wavelet_b200", "rl", "@", str(cfg)], cwd=ROOT, env=env,
                           capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-3000:]
        rows = [json.loads(line) for line in (tmp_path / "out" / "metrics.jsonl").read_text().splitlines()]
        assert [x["step"] for x in rows] == [1, 2]
        assert any("ref_kl" in k for k in rows[0]), sorted(rows[0])
    finally:
        os.killpg(srv.pid, 15)
        srv.wait(timeout=60)
