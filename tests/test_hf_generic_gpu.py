"""A generic Hugging Face architecture (Llama) on a B200: the transformers
module in bf16 (FlashAttention-2 varlen over packed documents when flash_attn
is installed), the CUDA chunked LM-head loss and fused AdamW steps."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_generic_llama_trains_on_gpu(cuda_ext):
    from wavelet_b200.data.fake import synthetic_sft_microbatches
    from wavelet_b200.models.config import resolve_arch
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.zero import AdamWHyper
    from wavelet_b200.trainer.engine import Engine

    cfg = resolve_arch("tiny-llama")
    m = build_model(cfg, "cuda", torch.bfloat16, seed=3)
    assert m.flat.compute.dtype == torch.bfloat16
    (b,) = synthetic_sft_microbatches(1, 256, cfg.vocab_size, seed=1, seqs_per_micro=3)
    b = b.to("cuda")
    # packed documents see only themselves
    h = m.hidden(b.input_ids, m.batch_ctx(b.position_ids, b.cu_seqlens, b.max_seqlen))
    s, e = int(b.cu_seqlens[1]), int(b.cu_seqlens[2])
    one = m.hidden(b.input_ids[s:e], m.batch_ctx(torch.arange(e - s, device="cuda"),
                                                 torch.tensor([0, e - s], dtype=torch.int32, device="cuda"), e - s))
    torch.testing.assert_close(h[s:e].float(), one.float(), rtol=2e-2, atol=2e-2)
    eng = Engine(m, AdamWHyper(lr=3e-3))
    scale = 1.0 / float(b.loss_mask.sum())
    losses = []
    for _ in range(5):
        losses.append(float(eng.sft_micro_step(b, scale)))
        eng.optimizer_step(3e-3)
    torch.cuda.synchronize()
    assert all(l == l for l in losses) and losses[-1] < losses[0], losses
    assert cuda_ext.read_error(0) == 0
