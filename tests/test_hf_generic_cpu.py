"""Architectures without a native decoder (Llama, Mistral, ...) through the
transformers module adapter: packed documents masked like separate runs, the
engine's loss equals the module's own cross entropy, tied embeddings stay one
store entry, training lowers the loss, HF-layout save / load round trips,
and the `sft` CLI trains a generic preset end to end."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from wavelet_b200.models.config import resolve_arch
from wavelet_b200.models.qwen import build_model
from wavelet_b200.parallel.zero import AdamWHyper
from wavelet_b200.trainer.engine import Engine


def _batch(cfg, seq=96, seed=1):
    from wavelet_b200.data.fake import synthetic_sft_microbatches

    (b,) = synthetic_sft_microbatches(1, seq, cfg.vocab_size, seed=seed, seqs_per_micro=3)
    return b


@pytest.mark.parametrize("name", ["tiny-llama", "tiny-mistral"])
def test_packed_rows_match_separate_documents(name):
    cfg = resolve_arch(name)
    m = build_model(cfg, "cpu", torch.float32, seed=0)
    b = _batch(cfg)
    h = m.hidden(b.input_ids, m.batch_ctx(b.position_ids, b.cu_seqlens, b.max_seqlen))
    cu = b.cu_seqlens.tolist()
    for s, e in zip(cu[:-1], cu[1:]):
        one = m.hidden(b.input_ids[s:e], m.batch_ctx(torch.arange(e - s), torch.tensor([0, e - s], dtype=torch.int32),
                                                      e - s))
        torch.testing.assert_close(h[s:e], one, rtol=1e-5, atol=1e-5)


def test_engine_loss_equals_module_cross_entropy_and_training_lowers_it():
    cfg = resolve_arch("tiny-llama")
    m = build_model(cfg, "cpu", torch.float32, seed=5)
    b = _batch(cfg, seed=2)
    n = float(b.loss_mask.sum())
    eng = Engine(m, AdamWHyper(lr=3e-3))
    first = float(eng.sft_micro_step(b, 1.0 / n))
    with torch.no_grad():
        logits = m.module(input_ids=b.input_ids[None], position_ids=b.position_ids[None].long(), use_cache=False).logits[0]
        ce = torch.nn.functional.cross_entropy(logits.float(), b.targets.clamp_min(0), reduction="none")
        want = float((ce * b.loss_mask * (b.targets >= 0)).sum() / n)
    assert abs(first - want) < 1e-4 * abs(want), (first, want)
    assert m.flat.grad.abs().sum() > 0
    eng.optimizer_step(3e-3)
    losses = [first]
    for _ in range(5):
        losses.append(float(eng.sft_micro_step(b, 1.0 / n)))
        eng.optimizer_step(3e-3)
    assert losses[-1] < losses[0], losses
    p = m.module.get_parameter("model.layers.0.mlp.down_proj.weight")
    assert p.data_ptr() == m.flat.view("model.layers.0.mlp.down_proj.weight").data_ptr()


def test_tied_embeddings_are_one_parameter():
    cfg = resolve_arch("tiny-mistral")
    assert cfg.tie_embeddings
    m = build_model(cfg, "cpu", torch.float32, seed=1)
    assert "lm_head.weight" not in m.flat.names() and m._head_name == "model.embed_tokens.weight"
    assert m.module.lm_head.weight is m.module.model.embed_tokens.weight
    eng = Engine(m, AdamWHyper(lr=1e-2))
    b = _batch(cfg)
    eng.sft_micro_step(b, 1.0 / float(b.loss_mask.sum()))
    eng.optimizer_step(1e-2)
    assert m.module.lm_head.weight.data_ptr() == m.flat.view("model.embed_tokens.weight").data_ptr()


def test_save_and_load_in_hf_layout(tmp_path):
    from transformers import AutoModelForCausalLM

    from wavelet_b200.models.hf_io import load_hf_weights, save_hf

    cfg = resolve_arch("tiny-llama")
    m = build_model(cfg, "cpu", torch.float32, seed=7)
    save_hf(m, tmp_path / "ck", dtype=torch.float32)
    assert json.loads((tmp_path / "ck" / "config.json").read_text())["model_type"] == "llama"
    # transformers reads it back as the same model
    back = AutoModelForCausalLM.from_pretrained(tmp_path / "ck").eval()
    ids = torch.tensor([[5, 6, 7, 8, 9]])
    with torch.no_grad():
        torch.testing.assert_close(back(ids).logits, m.module.eval()(ids).logits, rtol=1e-5, atol=1e-5)
    # and a fresh adapter loads it from the directory (resolve_arch on the path)
    cfg2 = resolve_arch(str(tmp_path / "ck"))
    assert getattr(cfg2, "generic_hf", False) and cfg2.source == str(tmp_path / "ck")
    m2 = build_model(cfg2, "cpu", torch.float32, seed=99)
    load_hf_weights(m2, tmp_path / "ck")
    for n in m.flat.names():
        torch.testing.assert_close(m2.flat.view(n), m.flat.view(n), rtol=0, atol=0)


def test_unsupported_heads_and_parallelism_are_refused():
    from wavelet_b200.models.hf_generic import HFGenericConfig

    with pytest.raises(NotImplementedError, match="soft"):
        HFGenericConfig({"model_type": "gemma2", "vocab_size": 10, "hidden_size": 8, "num_hidden_layers": 1,
                         "num_attention_heads": 1, "final_logit_softcapping": 30.0})
    with pytest.raises(NotImplementedError, match="data parallelism only"):
        build_model(resolve_arch("tiny-llama"), "cpu", torch.float32, tp=(2, 0))


def test_sft_cli_trains_a_generic_preset(tmp_path):
    root = Path(__file__).resolve().parents[1]
    out = tmp_path / "out"
    cfg = tmp_path / "sft.yaml"
    cfg.write_text((root / "examples" / "tiny_cpu" / "sft.yaml").read_text()
                   .replace("outputs/tiny_cpu_sft", str(out)).replace("name: tiny", "name: tiny-llama")
                   .replace("max_steps: 10", "max_steps: 3").replace("seq_len: 128", "seq_len: 64")
                   + "ckpt:\n  mode: async\n  interval: 3\n")
    env = {**os.environ, "WAVELET_FORCE_CPU": "1"}
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "sft", "@", str(cfg)], cwd=root, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    rows = [json.loads(line) for line in (out / "metrics.jsonl").read_text().splitlines()]
    assert [x["step"] for x in rows] == [1, 2, 3]
    assert (out / "checkpoint-3" / "STABLE").exists()


def test_hf_generator_greedy_stops_and_masks():
    """Rollouts for a generic model: greedy continuation equals step-by-step
    argmax of the module's own logits (left padding does not leak), stop
    tokens end a row after min_tokens, truncated sampling returns the kept
    token ids, and a seed makes sampling reproducible."""
    from wavelet_b200.inference.engine import SamplingParams
    from wavelet_b200.inference.hf_generator import HFGenerator, make_generator

    cfg = resolve_arch("tiny-llama")
    m = build_model(cfg, "cpu", torch.float32, seed=2)
    g = make_generator(m, max_num_seqs=4, max_model_len=64)
    assert isinstance(g, HFGenerator)
    prompts = [[5, 9, 13], [7, 3, 8, 11, 2, 4], [6]]
    out = g.generate(prompts, SamplingParams(temperature=0.0, max_tokens=6))
    for c in out:
        ids = list(c.prompt_ids)
        for t in c.token_ids:
            with torch.no_grad():
                want = int(m.module(input_ids=torch.tensor([ids]), use_cache=False).logits[0, -1].argmax())
            assert t == want
            ids.append(t)
        assert c.finish_reason == "length" and len(c.logprobs) == 6
    first = out[0].token_ids[1]
    stopped = g.generate([prompts[0]], SamplingParams(temperature=0.0, max_tokens=6, stop_token_ids=[first]))[0]
    assert stopped.token_ids == out[0].token_ids[:2] and stopped.finish_reason == "stop"
    held = g.generate([prompts[0]], SamplingParams(temperature=0.0, max_tokens=6, stop_token_ids=[first],
                                                   min_tokens=4))[0]
    assert len(held.token_ids) > 2
    p = SamplingParams(temperature=1.0, top_k=5, max_tokens=5, n=3, seed=11, return_sampling_mask=True)
    a, b = g.generate(prompts, p), g.generate(prompts, p)
    assert [c.token_ids for c in a] == [c.token_ids for c in b]
    assert all(len(mk) == 5 and t in mk for c in a for mk, t in zip(c.sampling_mask, c.token_ids))
    assert [(c.prompt_index, c.sample_index) for c in a] == [(i, j) for i in range(3) for j in range(3)]


def test_integrated_rl_trains_a_generic_model(tmp_path):
    root = Path(__file__).resolve().parents[1]
    cfg = tmp_path / "rl.yaml"
    cfg.write_text(f"""model:
  name: tiny-llama
  random_init: true
data:
  source: fake
  seq_len: 96
  fake_vocab_size: 64
  fake_prompt_len: 8
algo:
  type: grpo
reward:
  mode: reverse_match
orchestrator:
  examples_per_step: 2
  rollouts_per_example: 4
inference:
  sampling:
    max_completion_tokens: 8
lora: null
max_steps: 2
output_dir: {tmp_path / 'out'}
""")
    env = {**os.environ, "WAVELET_FORCE_CPU": "1"}
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "rl", "@", str(cfg)], cwd=root, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    rows = [json.loads(line) for line in (tmp_path / "out" / "metrics.jsonl").read_text().splitlines()]
    assert [x["step"] for x in rows] == [1, 2] and "reward/mean" in rows[0]
