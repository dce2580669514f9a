"""LoRA and QLoRA decoder on the GPU (LoRA-fused / NF4 tcgen05 GEMMs) against
the float32 CPU reference path with the same weights."""

from types import SimpleNamespace

import pytest
import torch

from wavelet_b200.data.fake import synthetic_sft_microbatches
from wavelet_b200.models.config import PRESETS
from wavelet_b200.models.qwen import build_model
from wavelet_b200.parallel.zero import AdamWHyper
from wavelet_b200.trainer.engine import Engine

pytestmark = pytest.mark.gpu

LORA = SimpleNamespace(rank=16, alpha=32.0, dropout=0.0,
                       target_modules=["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"])


@pytest.mark.parametrize("nf4", [False, True])
def test_lora_gpu_matches_cpu_reference(cuda_ext, nf4):
    cfg = PRESETS["tiny-gpu"]
    gpu = build_model(cfg, "cuda", torch.bfloat16, seed=3, lora=LORA, load_in_4bit=nf4)
    with torch.no_grad():  # non-zero B so every adapter path carries signal
        for n in gpu.lora.flat.names():
            if n.endswith(".B"):
                v = gpu.lora.flat.view(n)
                lay = gpu.lora.layouts[n.split(".")[1]]
                for _, _, lo, hi, c0 in lay.parts:
                    v[lo:hi, c0 : c0 + LORA.rank].normal_(0, 0.02)
        gpu.lora.flat.sync_master_from_compute()
    cpu = build_model(cfg, "cpu", torch.float32, init=False, lora=LORA, load_in_4bit=nf4)
    with torch.no_grad():
        cpu.flat.compute.copy_(gpu.flat.compute.float().cpu())
        cpu.lora.flat.compute.copy_(gpu.lora.flat.compute.float().cpu())
        for k, q in gpu.quant.items():
            cpu.quant[k].codes.copy_(q.codes.cpu())
            cpu.quant[k].absmax.copy_(q.absmax.cpu())
    (b,) = synthetic_sft_microbatches(1, 192, cfg.vocab_size, seed=1, seqs_per_micro=2)
    scale = 1.0 / float(b.loss_mask.sum())
    lg = Engine(gpu, AdamWHyper()).sft_micro_step(b.to("cuda"), scale)
    lc = Engine(cpu, AdamWHyper()).sft_micro_step(b, scale)
    torch.cuda.synchronize()
    assert cuda_ext.read_error(0) == 0
    assert abs(lg.item() - lc.item()) < 2e-2 * abs(lc.item()) + 1e-3, (lg.item(), lc.item())
    g_gpu, g_cpu = gpu.lora.flat.grad.cpu(), cpu.lora.flat.grad
    for name in cpu.lora.flat.names():
        off, n = cpu.lora.flat.offsets[name]
        a, r = g_gpu[off : off + n], g_cpu[off : off + n]
        cos = torch.nn.functional.cosine_similarity(a, r, dim=0).item()
        rel = ((a - r).norm() / (r.norm() + 1e-12)).item()
        assert cos > 0.99 and rel < 0.15, (name, cos, rel)


def test_qlora_training_reduces_loss(cuda_ext):
    cfg = PRESETS["tiny-gpu"]
    m = build_model(cfg, "cuda", torch.bfloat16, seed=0, lora=LORA, load_in_4bit=True)
    eng = Engine(m, AdamWHyper(lr=5e-3))
    (b,) = synthetic_sft_microbatches(1, 256, cfg.vocab_size, seed=0, seqs_per_micro=2)
    b = b.to("cuda")
    scale = 1.0 / float(b.loss_mask.sum())
    losses = []
    for _ in range(10):
        losses.append(eng.sft_micro_step(b, scale).item())
        eng.optimizer_step(5e-3)
    assert losses[-1] < losses[0] - 0.2, losses
