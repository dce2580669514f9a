"""The eager DeepSeek-V4 model on a B200: bf16 compute with the fp32
sensitive store, the CUDA chunked LM-head loss and fused AdamW steps."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_deepseek_v4_trains_on_gpu(cuda_ext):
    from wavelet_b200.data.fake import synthetic_sft_microbatches
    from wavelet_b200.models.config import resolve_arch
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.zero import AdamWHyper
    from wavelet_b200.trainer.engine import Engine

    cfg = resolve_arch("tiny-deepseek-v4")
    m = build_model(cfg, "cuda", torch.bfloat16, seed=3)
    assert m.flat.compute.dtype == torch.bfloat16 and m.expert_flat.compute.dtype == torch.float32
    assert m.module.model.layers[0].self_attn.sinks.dtype == torch.float32
    eng = Engine(m, AdamWHyper(lr=3e-3))
    (b,) = synthetic_sft_microbatches(1, 256, cfg.vocab_size, seed=1, seqs_per_micro=2)
    b = b.to("cuda")
    scale = 1.0 / float(b.loss_mask.sum())
    losses = []
    for _ in range(5):
        losses.append(float(eng.sft_micro_step(b, scale)))
        eng.optimizer_step(3e-3)
    torch.cuda.synchronize()
    assert all(l == l for l in losses) and losses[-1] < losses[0], losses
    assert cuda_ext.read_error(0) == 0
