"""The eager DeepSeek-V4 model through the trainer's engine: flat stores
(bf16 / fp32 split), gradients collected into them, sharded AdamW steps and
a decreasing loss on a repeated batch; the `sft` trainer runs it end to end
from a preset."""

import torch

from wavelet_b200.models.config import resolve_arch
from wavelet_b200.models.qwen import build_model
from wavelet_b200.parallel.zero import AdamWHyper
from wavelet_b200.trainer.engine import Engine


def test_engine_trains_deepseek_v4():
    from wavelet_b200.data.fake import synthetic_sft_microbatches

    cfg = resolve_arch("tiny-deepseek-v4")
    m = build_model(cfg, "cpu", torch.float32, seed=3)
    assert m.expert_flat.compute.dtype == torch.float32
    assert "model.layers.0.self_attn.sinks" in m.expert_flat.names()
    assert "lm_head.weight" in m.flat.names()
    eng = Engine(m, AdamWHyper(lr=3e-3))
    (b,) = synthetic_sft_microbatches(1, 96, cfg.vocab_size, seed=1, seqs_per_micro=2)
    scale = 1.0 / float(b.loss_mask.sum())
    losses = []
    for _ in range(6):
        losses.append(float(eng.sft_micro_step(b, scale)))
        assert m.flat.grad.abs().sum() > 0 and m.expert_flat.grad.abs().sum() > 0
        eng.optimizer_step(3e-3)
    assert losses[-1] < losses[0], losses
    # module parameters are views of the stores: an optimizer step moved them
    p = dict(m.module.named_parameters())["lm_head.weight"]
    assert p.data_ptr() == m.flat.view("lm_head.weight").data_ptr()


def test_engine_loss_matches_module_loss():
    from wavelet_b200.data.fake import synthetic_sft_microbatches
    from wavelet_b200.ops import reference as ref  # noqa: F401

    cfg = resolve_arch("tiny-deepseek-v4")
    m = build_model(cfg, "cpu", torch.float32, seed=5)
    (b,) = synthetic_sft_microbatches(1, 64, cfg.vocab_size, seed=2, seqs_per_micro=1)
    n = float(b.loss_mask.sum())
    loss = float(Engine(m, AdamWHyper()).sft_micro_step(b, 1.0 / n))
    with torch.no_grad():
        logits = m.module.lm_head(m.module.model(b.input_ids, (b.cu_seqlens[1:] - b.cu_seqlens[:-1]).long()))
        ce = torch.nn.functional.cross_entropy(logits.float(), b.targets.clamp_min(0), reduction="none")
        want = float((ce * b.loss_mask * (b.targets >= 0)).sum() / n)
    assert abs(loss - want) < 1e-4 * abs(want), (loss, want)


def test_sft_cli_trains_deepseek_v4(tmp_path):
    import json
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    out = tmp_path / "out"
    cfg = tmp_path / "sft.yaml"
    cfg.write_text((root / "examples" / "tiny_cpu" / "sft.yaml").read_text()
                   .replace("outputs/tiny_cpu_sft", str(out)).replace("name: tiny", "name: tiny-deepseek-v4")
                   .replace("max_steps: 10", "max_steps: 4").replace("seq_len: 128", "seq_len: 64")
                   + "ckpt:\n  mode: async\n  interval: 4\n")
    env = {**os.environ, "WAVELET_FORCE_CPU": "1"}
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "sft", "@", str(cfg)], cwd=root, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    rows = [json.loads(line) for line in (out / "metrics.jsonl").read_text().splitlines()]
    assert [x["step"] for x in rows] == [1, 2, 3, 4]
    assert (out / "checkpoint-4" / "STABLE").exists()


def test_trainer_checkpoint_converts_to_native(tmp_path):
    """checkpoint-N of a DeepSeek-V4 SFT run -> native checkpoint whose
    logits equal the trained model's."""
    from wavelet_b200.models.deepseek_v4 import DeepseekV4ForCausalLM
    from wavelet_b200.tools.convert_checkpoint import convert_checkpoint
    from wavelet_b200.trainer.ckpt import CheckpointManager

    cfg = resolve_arch("tiny-deepseek-v4")
    m = build_model(cfg, "cpu", torch.float32, seed=9)
    eng = Engine(m, AdamWHyper(lr=1e-3))
    with torch.no_grad():  # routing state lives in buffers, outside the flat stores
        m.module.model.layers[0].mlp.router.tid2eid.copy_(torch.randint(0, 4, (1024, 2)))
        m.module.model.layers[1].mlp.router.selection_bias.uniform_(-0.1, 0.1)
    mgr = CheckpointManager(tmp_path / "ckpts", mode="async")
    d = mgr.save(1, model=m, optimizer=eng.opt, data_state=None, meta={"arch": cfg.to_dict()}, block=True)
    mgr.wait()
    out = convert_checkpoint(d, tmp_path / "native", dtype="float32")
    back = DeepseekV4ForCausalLM.from_pretrained(out).eval()
    ids = torch.tensor([[5, 6, 7, 8, 9, 10, 11, 12]])
    with torch.no_grad():
        torch.testing.assert_close(back(ids).logits, m.module.eval()(ids).logits, atol=1e-6, rtol=1e-6)
