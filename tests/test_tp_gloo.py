"""Tensor parallelism (Megatron split of every decoder layer, row-parallel
partial sums all-reduced) on 2 gloo CPU ranks against the unsplit model: the
loss and every rank's local gradient slice match."""

import os
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _batch(cfg):
    from wavelet_b200.data.fake import synthetic_sft_microbatches

    (b,) = synthetic_sft_microbatches(1, 64, cfg.vocab_size, seed=2, seqs_per_micro=2)
    return b


def _worker(rank, world, init_file, out):
    os.environ["WAVELET_FORCE_CPU"] = "1"
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.zero import AdamWHyper
    from wavelet_b200.trainer.engine import Engine

    cfg = PRESETS["tiny"]
    m = build_model(cfg, "cpu", torch.float32, seed=9, tp=(world, rank))
    m.tp_group = dist.group.WORLD
    b = _batch(cfg)
    loss = Engine(m, AdamWHyper()).sft_micro_step(b, 1.0 / float(b.loss_mask.sum()))
    m.finalize_grads()
    torch.save({"loss": float(loss), "grads": {n: m.flat.grad_view(n).clone() for n in m.flat.names()}},
               f"{out}.{rank}")
    dist.destroy_process_group()


def test_tp2_matches_unsplit():
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model, tp_slicers
    from wavelet_b200.parallel.zero import AdamWHyper
    from wavelet_b200.trainer.engine import Engine

    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(world, os.path.join(d, "init"), os.path.join(d, "res")), nprocs=world, join=True)
        got = [torch.load(os.path.join(d, f"res.{r}")) for r in range(world)]
    cfg = PRESETS["tiny"]
    ref = build_model(cfg, "cpu", torch.float32, seed=9)
    ref.fused_cpu = True
    b = _batch(cfg)
    loss = Engine(ref, AdamWHyper()).sft_micro_step(b, 1.0 / float(b.loss_mask.sum()))
    for r in range(world):
        assert abs(got[r]["loss"] - float(loss)) < 1e-4 * abs(float(loss)) + 1e-6
        sl = tp_slicers(cfg, world, r)
        for n, g in got[r]["grads"].items():
            full = ref.flat.grad_view(n)
            key = n.split(".", 1)[-1]
            want = sl[key][1](full) if key in sl else full
            torch.testing.assert_close(g, want, rtol=1e-4, atol=1e-6, msg=n)


def _norm_worker(rank, world, init_file, out):
    os.environ["WAVELET_FORCE_CPU"] = "1"
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.zero import AdamWHyper
    from wavelet_b200.trainer.engine import Engine

    cfg = PRESETS["tiny"]
    m = build_model(cfg, "cpu", torch.float32, seed=9, tp=(world, rank))
    m.tp_group = dist.group.WORLD
    b = _batch(cfg)
    eng = Engine(m, AdamWHyper(max_grad_norm=0.5))
    eng.sft_micro_step(b, 1.0 / float(b.loss_mask.sum()))
    st = eng.optimizer_step(1e-3)
    torch.save({"norm": st["grad_norm"], "factor": st["clip_factor"]}, f"{out}.{rank}")
    dist.destroy_process_group()


def test_tp2_grad_norm_counts_replicated_params_once():
    """Under TP the optimizer's global gradient norm sums the split weights
    over the TP ranks and the replicated ones (embeddings, norms, LM head)
    once: it equals the unsplit model's norm, and so does the clip factor."""
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model
    from wavelet_b200.parallel.zero import AdamWHyper
    from wavelet_b200.trainer.engine import Engine

    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_norm_worker, args=(world, os.path.join(d, "init"), os.path.join(d, "res")), nprocs=world,
                 join=True)
        got = [torch.load(os.path.join(d, f"res.{r}")) for r in range(world)]
    cfg = PRESETS["tiny"]
    ref = build_model(cfg, "cpu", torch.float32, seed=9)
    ref.fused_cpu = True
    b = _batch(cfg)
    eng = Engine(ref, AdamWHyper(max_grad_norm=0.5))
    eng.sft_micro_step(b, 1.0 / float(b.loss_mask.sum()))
    st = eng.optimizer_step(1e-3)
    for r in range(world):
        assert abs(got[r]["norm"] - st["grad_norm"]) <= 1e-4 * st["grad_norm"], (got[r]["norm"], st["grad_norm"])
        assert abs(got[r]["factor"] - st["clip_factor"]) <= 1e-4
