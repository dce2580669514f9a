"""Tensor-parallel generation over 2 gloo ranks: a TP2 split of the model
(heads and FFN columns per rank, row-parallel outputs all-reduced) decodes
the same greedy tokens as the unsplit model, and sampled tokens agree on
both TP ranks without a fixed seed (the group shares one); greedy decoding
on the CPU path is an argmax."""

import os
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

PROMPTS = [[5, 9, 13, 2, 7], [3, 3, 8], [11, 4, 6, 1, 9, 12, 2]]


def _gen(model):
    from wavelet_b200.inference.engine import Generator

    return Generator(model, max_num_seqs=8, max_model_len=64, kv_cache_bytes=None, block_size=16)


def _worker(rank, world, init_file, res):
    os.environ["WAVELET_FORCE_CPU"] = "1"
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    from wavelet_b200.inference.engine import SamplingParams
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model

    cfg = PRESETS["tiny"]
    m = build_model(cfg, "cpu", torch.float32, seed=4, tp=(world, rank), with_grad=False, with_optimizer=False)
    m.tp_group = dist.group.WORLD
    g = _gen(m)
    assert g.k_cache[0].shape[1] == cfg.num_kv_heads // world
    greedy = g.generate(PROMPTS, SamplingParams(temperature=0.0, max_tokens=12, n=1))
    sampled = g.generate(PROMPTS, SamplingParams(temperature=1.0, max_tokens=12, n=2, seed=None))
    out = {"greedy": [c.token_ids for c in greedy], "sampled": [c.token_ids for c in sampled],
           "lp": [c.logprobs for c in greedy]}
    torch.save(out, f"{res}.{rank}")
    dist.barrier()
    dist.destroy_process_group()
    os._exit(0)  # results are on disk; skip gloo's interpreter teardown


def test_tp2_generation_matches_unsplit_model():
    os.environ["WAVELET_FORCE_CPU"] = "1"
    from wavelet_b200.inference.engine import SamplingParams
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model

    with tempfile.TemporaryDirectory() as d:
        res = os.path.join(d, "res")
        mp.spawn(_worker, args=(2, os.path.join(d, "init"), res), nprocs=2, join=True)
        r0, r1 = torch.load(f"{res}.0"), torch.load(f"{res}.1")
    assert r0["greedy"] == r1["greedy"] and r0["sampled"] == r1["sampled"]  # the TP ranks agree
    full = build_model(PRESETS["tiny"], "cpu", torch.float32, seed=4, with_grad=False, with_optimizer=False)
    ref = _gen(full).generate(PROMPTS, SamplingParams(temperature=0.0, max_tokens=12, n=1))
    assert [c.token_ids for c in ref] == r0["greedy"]
    for a, b in zip([c.logprobs for c in ref], r0["lp"]):
        torch.testing.assert_close(torch.tensor(b), torch.tensor(a), rtol=1e-4, atol=1e-4)
    assert all(len(t) == 12 for t in r0["greedy"])


def test_integrated_rl_with_tp2_trainer_and_generator(tmp_path):
    """`wavelet rl` (integrated) on 2 gloo ranks with fsdp.tp=2: the TP-split
    model generates (once per TP group) and trains."""
    import json
    import socket
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
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
  type: grpo
reward:
  mode: reverse_match
orchestrator:
  examples_per_step: 4
  rollouts_per_example: 4
inference:
  sampling:
    max_completion_tokens: 8
fsdp:
  backend: gloo
  tp: 2
lora: null
max_steps: 2
output_dir: {tmp_path / 'out'}
""")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = {**os.environ, "WAVELET_FORCE_CPU": "1"}
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "wavelet_b200", "rl", "@",
                        str(cfg)], cwd=root, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    rows = [json.loads(line) for line in (tmp_path / "out" / "metrics.jsonl").read_text().splitlines()]
    assert [x["step"] for x in rows] == [1, 2]
    # one copy of each rollout: 4 prompts x 4 samples per step, not doubled by the TP peer
    assert all(0 < x["train/num_samples"] <= 16 for x in rows)
