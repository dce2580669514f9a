"""A vision-language model (Qwen2.5-VL layout) on a B200: documents with
images through the transformers module in bf16, the CUDA chunked LM-head
loss and fused AdamW steps."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_vlm_trains_on_gpu(cuda_ext):
    import importlib.util
    import os

    spec = importlib.util.spec_from_file_location("vlm_cpu_rows", os.path.join(os.path.dirname(__file__),
                                                                              "test_vlm_cpu.py"))
    rows = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rows)
    _batch, _row = rows._batch, rows._row
    from wavelet_b200.models.config import resolve_arch
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.zero import AdamWHyper
    from wavelet_b200.trainer.engine import Engine

    m = build_model(resolve_arch("tiny-qwen2.5-vl"), "cuda", torch.bfloat16, seed=3)
    b = _batch([_row(1, 1), _row(2, 0), _row(3, 2)]).to("cuda")
    eng = Engine(m, AdamWHyper(lr=3e-3))
    n = float(b.loss_mask.sum())
    losses = []
    for _ in range(5):
        losses.append(float(eng.sft_micro_step(b, 1.0 / n)))
        eng.optimizer_step(3e-3)
    torch.cuda.synchronize()
    assert all(l == l for l in losses) and losses[-1] < losses[0], losses
    assert cuda_ext.read_error(0) == 0
