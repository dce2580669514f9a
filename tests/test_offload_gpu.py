"""Activation offloading (layer inputs in pinned host memory) and optimizer
state offloading (chunked host <-> device AdamW) give the results of the
device-resident runs."""

import pytest
import torch

from wavelet_b200.data.fake import synthetic_sft_microbatches
from wavelet_b200.models.config import PRESETS
from wavelet_b200.models.qwen import build_model
from wavelet_b200.parallel.zero import AdamWHyper, ShardedAdamW
from wavelet_b200.trainer.engine import Engine

pytestmark = pytest.mark.gpu


def test_activation_offload_matches(cuda_ext):
    cfg = PRESETS["tiny-gpu"]
    (b,) = synthetic_sft_microbatches(1, 4096, cfg.vocab_size, seed=1, seqs_per_micro=2)  # layer input > 2 MB
    b = b.to("cuda")
    grads = []
    for off in (False, True):
        m = build_model(cfg, "cuda", torch.bfloat16, seed=3)
        m.enable_activation_offload(off)
        Engine(m, AdamWHyper()).sft_micro_step(b, 1e-3)
        torch.cuda.synchronize()
        grads.append(m.flat.grad.clone())
    # the restored layer inputs are bit-exact; the norm-weight and embedding
    # gradients accumulate with float atomics, so only their summation order varies
    torch.testing.assert_close(grads[0], grads[1], rtol=1e-4, atol=1e-6)


def test_optimizer_offload_matches(cuda_ext):
    cfg = PRESETS["tiny-gpu"]
    ms = [build_model(cfg, "cuda", torch.bfloat16, seed=4) for _ in range(2)]
    h = AdamWHyper(lr=1e-3, weight_decay=0.01)
    opts = [ShardedAdamW(ms[0].flat, h), ShardedAdamW(ms[1].flat, h, offload=True, offload_chunk=100_000)]
    assert ms[1].flat.master.device.type == "cpu" and ms[1].flat.master.is_pinned()
    for it in range(3):
        g = torch.randn(ms[0].flat.numel, device="cuda") * (it + 1)
        for m, o in zip(ms, opts):
            m.flat.grad.copy_(g)
            o.step()
    torch.cuda.synchronize()
    assert torch.equal(ms[0].flat.compute, ms[1].flat.compute)
    assert torch.equal(ms[0].flat.master.cpu(), ms[1].flat.master)


def test_kept_activations_match_recompute(cuda_ext):
    cfg = PRESETS["tiny-gpu"]
    (b,) = synthetic_sft_microbatches(1, 512, cfg.vocab_size, seed=5, seqs_per_micro=2)
    b = b.to("cuda")
    grads = []
    for every in (1, None, 2):
        m = build_model(cfg, "cuda", torch.bfloat16, seed=6)
        m.set_activation_checkpointing(every)
        Engine(m, AdamWHyper()).sft_micro_step(b, 1e-3)
        torch.cuda.synchronize()
        grads.append(m.flat.grad.clone())
    # same kernels on the same activations; only the float-atomic summation
    # order of the norm-weight / embedding gradients can differ
    for g in grads[1:]:
        torch.testing.assert_close(grads[0], g, rtol=1e-4, atol=1e-6)
