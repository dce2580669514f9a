"""The fused GPU decoder (kernels + recompute backward) against the float32
CPU reference path of the same model with the same weights."""

import pytest
import torch

from wavelet_b200.data.fake import synthetic_sft_microbatches
from wavelet_b200.models.config import PRESETS
from wavelet_b200.models.qwen import build_model
from wavelet_b200.parallel.zero import AdamWHyper
from wavelet_b200.trainer.engine import Engine

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("preset", ["tiny-gpu", "tiny-qwen2-gpu"])
def test_gpu_model_matches_cpu_reference(cuda_ext, preset):
    cfg = PRESETS[preset]
    gpu = build_model(cfg, "cuda", torch.bfloat16, seed=3)
    # give biases non-trivial values
    for n in gpu.flat.names():
        if n.endswith("qkv_b"):
            gpu.flat.view(n).normal_(0, 0.02)
    cpu = build_model(cfg, "cpu", torch.float32, init=False)
    with torch.no_grad():
        cpu.flat.compute.copy_(gpu.flat.compute.float().cpu())
    (b,) = synthetic_sft_microbatches(1, 192, cfg.vocab_size, seed=1, seqs_per_micro=2)
    scale = 1.0 / float(b.loss_mask.sum())
    eg = Engine(gpu, AdamWHyper())
    ec = Engine(cpu, AdamWHyper())
    lg = eg.sft_micro_step(b.to("cuda"), scale)
    lc = ec.sft_micro_step(b, scale)
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) == 0
    assert abs(lg.item() - lc.item()) < 2e-2 * abs(lc.item()) + 1e-3, (lg.item(), lc.item())
    g_gpu = gpu.flat.grad.cpu()
    g_cpu = cpu.flat.grad
    for name in cpu.flat.names():
        off, n = cpu.flat.offsets[name]
        a, r = g_gpu[off : off + n], g_cpu[off : off + n]
        cos = torch.nn.functional.cosine_similarity(a, r, dim=0).item()
        rel = ((a - r).norm() / (r.norm() + 1e-12)).item()
        assert cos > 0.99 and rel < 0.15, (name, cos, rel)


def test_gpu_training_reduces_loss(cuda_ext):
    cfg = PRESETS["tiny-gpu"]
    m = build_model(cfg, "cuda", torch.bfloat16, seed=0)
    eng = Engine(m, AdamWHyper(lr=3e-3))
    (b,) = synthetic_sft_microbatches(1, 256, cfg.vocab_size, seed=0, seqs_per_micro=2)
    b = b.to("cuda")
    scale = 1.0 / float(b.loss_mask.sum())
    losses = []
    for _ in range(8):
        losses.append(eng.sft_micro_step(b, scale).item())
        eng.optimizer_step(3e-3)
    assert losses[-1] < losses[0] - 0.5, losses
