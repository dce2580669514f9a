"""Expert-parallel MoE block (dispatch / combine over all-to-all) on 2 gloo
CPU ranks against the single-rank block with all experts and the same
weights: outputs, input gradients and router/norm gradients per rank, and
expert gradients summed over both ranks' tokens."""

import os
import tempfile

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _tokens(rank, T=37, H=128):
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randn(T, H, generator=g), torch.randn(T, H, generator=g)


def _worker(rank, world, init_file, out):
    os.environ["WAVELET_FORCE_CPU"] = "1"
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model

    cfg = PRESETS["tiny-moe"]
    m = build_model(cfg, "cpu", torch.float32, seed=7, ep=(world, rank, 0, 1))
    layer = m.layers[0]
    blk = layer.moe
    blk.ep_group = dist.group.WORLD
    x2, dout = _tokens(rank)
    y, cache = blk.forward(x2, layer.P, save=True)
    dx = blk.backward(dout, x2, cache, layer.P, layer.G)
    res = {"y": y, "dx": dx, "router": layer.G["router_w"].clone(), "norm": layer.G["post_norm"].clone(),
           "gu": layer.G["exp_gu_w"].clone(), "down": layer.G["exp_down_w"].clone()}
    torch.save(res, f"{out}.{rank}")
    dist.destroy_process_group()


def test_ep2_matches_single_rank():
    from wavelet_b200.models.config import PRESETS
    from wavelet_b200.models.qwen import build_model

    world = 2
    with tempfile.TemporaryDirectory() as d:
        init = os.path.join(d, "init")
        out = os.path.join(d, "res")
        mp.spawn(_worker, args=(world, init, out), nprocs=world, join=True)
        got = [torch.load(f"{out}.{r}") for r in range(world)]
    cfg = PRESETS["tiny-moe"]
    ref = build_model(cfg, "cpu", torch.float32, seed=7)
    layer = ref.layers[0]
    blk = layer.moe
    El = cfg.num_experts // world
    for r in range(world):
        x2, dout = _tokens(r)
        ref.flat.zero_grad()
        y, cache = blk.forward(x2, layer.P, save=True)
        dx = blk.backward(dout, x2, cache, layer.P, layer.G)
        torch.testing.assert_close(got[r]["y"], y, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(got[r]["dx"], dx, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(got[r]["router"], layer.G["router_w"], rtol=1e-4, atol=1e-6)
        torch.testing.assert_close(got[r]["norm"], layer.G["post_norm"], rtol=1e-4, atol=1e-6)
    # expert gradients: sum over both ranks' tokens, rank r holds experts [r*El, (r+1)*El)
    ref.flat.zero_grad()
    for r in range(world):
        x2, dout = _tokens(r)
        y, cache = blk.forward(x2, layer.P, save=True)
        blk.backward(dout, x2, cache, layer.P, layer.G)
    for r in range(world):
        torch.testing.assert_close(got[r]["gu"], layer.G["exp_gu_w"][r * El : (r + 1) * El], rtol=1e-4, atol=1e-6)
        torch.testing.assert_close(got[r]["down"], layer.G["exp_down_w"][r * El : (r + 1) * El], rtol=1e-4, atol=1e-6)
