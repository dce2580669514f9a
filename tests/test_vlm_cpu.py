"""Vision-language SFT through the transformers module adapter (Qwen2.5-VL
layout): pre-tokenized rows with processor image fields pack into rows whose
documents carry their images; the engine's loss equals the module's own
cross entropy on each document with its pixels; images change the loss;
training lowers it; a text-only model refuses image inputs; the `sft` CLI
trains from a JSONL of such rows."""

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

IMG, VS, VE = 1000, 1002, 1003


def _row(seed: int, n_images: int, text: int = 12) -> dict:
    """One document: text, then per image <vision_start> 1 image token <vision_end>
    (a 28x28 image: grid (1, 2, 2) = 4 patches of 3*2*14*14 values, merged 2x2)."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(3, 900, (text,), generator=g).tolist()
    for _ in range(n_images):
        ids += [VS, IMG, VE] + torch.randint(3, 900, (4,), generator=g).tolist()
    mm = None
    if n_images:
        mm = {"pixel_values": torch.randn(4 * n_images, 3 * 2 * 14 * 14, generator=g).tolist(),
              "image_grid_thw": [[1, 2, 2]] * n_images}
    return {"input_ids": ids, "loss_mask": [0] * 4 + [1] * (len(ids) - 4), **({"mm_kwargs": mm} if mm else {})}


def _batch(rows):
    from wavelet_b200.data.sft import _pretokenized, pack

    ss = [_pretokenized(r) for r in rows]
    return pack([torch.tensor(s.input_ids) for s in ss], [torch.tensor(s.loss_mask, dtype=torch.float32) for s in ss],
                [s.mm for s in ss])


def test_packed_images_and_loss_parity():
    cfg = resolve_arch("tiny-qwen2.5-vl")
    m = build_model(cfg, "cpu", torch.float32, seed=3)
    rows = [_row(1, 1), _row(2, 0), _row(3, 2)]
    b = _batch(rows)
    assert b.mm["doc_images"] == [1, 0, 2] and b.mm["pixel_values"].shape[0] == 12
    n = float(b.loss_mask.sum())
    loss = float(Engine(m, AdamWHyper()).sft_micro_step(b, 1.0 / n))
    want, cu = 0.0, b.cu_seqlens.tolist()
    with torch.no_grad():
        pi = 0
        for d, r in enumerate(rows):
            ids = torch.tensor([r["input_ids"]])
            kw = {}
            if r.get("mm_kwargs"):
                k = len(r["mm_kwargs"]["image_grid_thw"])
                kw = {"pixel_values": b.mm["pixel_values"][pi:pi + 4 * k],
                      "image_grid_thw": torch.tensor(r["mm_kwargs"]["image_grid_thw"])}
                pi += 4 * k
            logits = m.module(input_ids=ids, use_cache=False, **kw).logits[0]
            s, e = cu[d], cu[d + 1]
            ce = torch.nn.functional.cross_entropy(logits.float(), b.targets[s:e].clamp_min(0), reduction="none")
            want += float((ce * b.loss_mask[s:e]).sum())
    want /= n
    assert abs(loss - want) < 1e-4 * abs(want), (loss, want)
    # the pixels matter
    b2 = _batch(rows)
    b2.mm["pixel_values"] = b2.mm["pixel_values"] * 0 + 1
    m.flat.zero_grad()
    loss2 = float(Engine(m, AdamWHyper()).sft_micro_step(b2, 1.0 / n))
    assert abs(loss2 - loss) > 1e-5


def test_training_lowers_the_loss_and_text_models_refuse_images():
    cfg = resolve_arch("tiny-qwen2.5-vl")
    m = build_model(cfg, "cpu", torch.float32, seed=5)
    b = _batch([_row(7, 1), _row(8, 1)])
    eng = Engine(m, AdamWHyper(lr=3e-3))
    n = float(b.loss_mask.sum())
    losses = []
    for _ in range(5):
        losses.append(float(eng.sft_micro_step(b, 1.0 / n)))
        eng.optimizer_step(3e-3)
    assert losses[-1] < losses[0], losses
    text = build_model(resolve_arch("tiny-llama"), "cpu", torch.float32, seed=1)
    with pytest.raises(ValueError, match="vision tower"):
        Engine(text, AdamWHyper()).sft_micro_step(b, 1.0 / n)
    from wavelet_b200.data.sft import Sample, _check_fits

    with pytest.raises(ValueError, match="image"):
        _check_fits(Sample([1] * 10, [1] * 10, mm={"pixel_values": torch.zeros(1)}), 8)


def test_sft_cli_trains_a_vision_language_model(tmp_path):
    root = Path(__file__).resolve().parents[1]
    data = tmp_path / "vl.jsonl"
    data.write_text("".join(json.dumps(_row(i, i % 3)) + "\n" for i in range(8)))
    out = tmp_path / "out"
    cfg = tmp_path / "sft.yaml"
    cfg.write_text(f"""model:
  name: tiny-qwen2.5-vl
  random_init: true
data:
  source: local
  path: {data}
  seq_len: 64
  batch_size: 4
  micro_batch_size: 2
max_steps: 2
lora: null
optim:
  lr: 1e-3
output_dir: {out}
monitor:
  wandb:
    enabled: false
""")
    env = {**os.environ, "WAVELET_FORCE_CPU": "1"}
    r = subprocess.run([sys.executable, "-m", "wavelet_b200", "sft", "@", str(cfg)], cwd=root, env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    rows = [json.loads(line) for line in (out / "metrics.jsonl").read_text().splitlines()]
    assert [x["step"] for x in rows] == [1, 2]


def test_frozen_vision_encoder_stays_put():
    """model.vlm.freeze_vision_encoder: the vision tower keeps its weights
    through optimizer steps (weight decay included) while the decoder moves."""
    from types import SimpleNamespace

    from wavelet_b200.trainer.model_options import apply_model_options

    m = build_model(resolve_arch("tiny-qwen2.5-vl"), "cpu", torch.float32, seed=5)
    mcfg = SimpleNamespace(vlm=SimpleNamespace(freeze_vision_encoder=True, vision_encoder_attr="model.visual"))
    notes = apply_model_options(m, mcfg)
    assert any("vision-tower parameters frozen" in n for n in notes)
    before = {n: m.flat.view(n).clone() for n in m.flat.names()}
    eng = Engine(m, AdamWHyper(lr=3e-3, weight_decay=0.1))
    b = _batch([_row(7, 1), _row(8, 1)])
    for _ in range(2):
        eng.sft_micro_step(b, 1.0 / float(b.loss_mask.sum()))
        eng.optimizer_step(3e-3)
    vis = [n for n in m.flat.names() if n.startswith("model.visual.")]
    assert vis and all(torch.equal(m.flat.view(n), before[n]) for n in vis)
    assert not torch.equal(m.flat.view("lm_head.weight"), before["lm_head.weight"])
